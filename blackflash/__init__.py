"""Drop-in import path of the reference (`from blackflash import blackflash`,
reference blackflash/__init__.py:5-18), served by blackflash_b200."""
from blackflash_b200 import blackflash  # noqa: F401

__all__ = ["blackflash"]
