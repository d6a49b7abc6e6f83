// C++ launch interface kept signature-identical to the reference's
// include/flash_attn.cuh:22-32, so a caller written against the reference
// (its src/main.cu harness, or binding/blackflash_ops.cu:6-16) links against
// libblackflash_b200.so without source changes.
//
// Arguments: Q, K, V, O are [B, H, N, d] bf16 device tensors; l and m are
// [B, H, N] fp32 and receive the logsumexp and the row max of scale*QK^T
// (either may be null); d must be 64 (or 128, an extension). The call is asynchronous on `stream`.
// Unlike the reference it never calls exit(): on an error it prints the
// message to stderr and leaves it in blackflash_last_error() (blackflash_b200.h).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "blackflash_b200.h"

void flash_attn_naive_launch(const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V,
                             __nv_bfloat16* O, float* l, float* m, int B, int H, int N, int d, float scale,
                             cudaStream_t stream = 0);
