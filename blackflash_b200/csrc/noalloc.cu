// blackflash_bwd_noalloc: the attention backward for callers that cannot allocate
// device memory. Some hosts own every byte of device memory and give a plugin no
// way to call cudaMalloc (an inference server or framework that reserves its pool
// up front), and some loops cannot afford cudaMalloc / cudaFree, which may
// synchronise the device. blackflash_bwd needs a workspace from its caller; this
// entry point uses a fixed array compiled into the library instead.
//
// The array is a file-scope __device__ variable, so every GPU that loads the
// library holds it (kNoAllocScratchBytes) until the process exits. Host code may
// not pass the array's name to a kernel: on the host that name is only a stand-in
// for the symbol, not a device address. The device address is looked up with
// cudaGetSymbolAddress once per device, with that device current, on the first
// call made on that device; make that first call before any stream capture. The
// address is kept for the life of the process: after cudaDeviceReset (or any other
// teardown of the device's primary context) it is stale, so a process that resets a
// device must not call this entry point on it again.
//
// Every call on a device shares the one array and finds the previous call's data
// in it. The backward clears the part that must start at zero (the fp32 dQ
// accumulator, by a memset on the caller's stream) and overwrites the rest, so
// calls in sequence on one stream are safe; calls that overlap on the GPU (other
// streams, other threads) race on the array.
#include <cuda_runtime.h>
#include <string.h>

#include <mutex>

#include "fa_fwd_sm100.h"

namespace {

constexpr long long kNoAllocScratchBytes = 64LL << 20;  // 64 MiB per device

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_ptr[64] = {nullptr};

}  // namespace

extern "C" int blackflash_bwd_noalloc(const void* Q, const void* K, const void* V, const void* O, const void* dO,
                                      const float* lse, void* dQ, void* dK, void* dV, int B, int H, int N, int d,
                                      float scale, void* stream) {
    bf_set_error(BF_OK, "");  // clear the calling thread's last error, as every entry point does
    if (B <= 0 || H <= 0 || N <= 0) return bf_set_error(BF_ERR_ARG, "empty problem: B, H and N must be >= 1");
    if (d != 64) return bf_set_error(BF_ERR_ARG, "the backward supports d=64");
    const long long need = bf_bwd_workspace_bytes((long long)B * H, N);
    if (need > kNoAllocScratchBytes)
        return bf_set_error(BF_ERR_ARG,
                            "blackflash_bwd_noalloc: problem needs more than its fixed 64 MiB scratch "
                            "(B*H*N at most about 250000 rows); use blackflash_bwd with a workspace");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return bf_set_error(BF_ERR_CUDA, "cudaGetDevice failed");
    void* scratch;
    {
        std::lock_guard<std::mutex> lock(g_setup_mu);
        if (!g_scratch_ptr[dev]) {
            void* ptr = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
            if (e != cudaSuccess || !ptr) return bf_set_error(BF_ERR_CUDA, cudaGetErrorString(e));
            g_scratch_ptr[dev] = ptr;
        }
        scratch = g_scratch_ptr[dev];
    }
    BfBwdArgs a;
    memset(&a, 0, sizeof(a));
    a.q = Q;
    a.k = K;
    a.v = V;
    a.o = O;
    a.dout = dO;
    a.lse = lse;
    a.dq = dQ;
    a.dk = dK;
    a.dv = dV;
    a.workspace = scratch;
    a.bh = (long long)B * H;
    a.n = N;
    a.d = d;
    a.scale = scale;
    a.stream = stream;
    return bf_bwd_launch(&a);
}
