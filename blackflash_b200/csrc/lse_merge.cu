// Log-sum-exp merge of partial attention results (ring / sequence-parallel
// mode) and the final fp32 -> bf16 cast. Both are HBM-bound streaming kernels:
// each fp32 element is read twice and written once (merge), or read once and
// written as bf16 (cast). Sixteen threads cover one 64-wide row with float4
// accesses, so a warp touches two full rows (512 contiguous bytes per array).
#include <cuda_bf16.h>
#include <math.h>

#include "fa_fwd_sm100.h"

namespace bfk {

__global__ void lse_merge_kernel(float4* __restrict__ o_acc, float* __restrict__ lse_acc,
                                 const float4* __restrict__ o_part, const float* __restrict__ lse_part,
                                 long long rows) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // float4 index
    const long long row = i >> 4;
    const bool live = row < rows;
    float la = -INFINITY, lp = -INFINITY;
    if (live) {
        la = lse_acc[row];
        lp = lse_part[row];
    }
    __syncwarp();  // all 16 lanes of the row have read lse_acc before lane 0 rewrites it
    if (!live) return;
    const float m = fmaxf(la, lp);
    if (m == -INFINITY) return;  // both empty: nothing to do
    const float wa = expf(la - m);
    const float wp = expf(lp - m);
    const float inv = 1.f / (wa + wp);
    const float ca = wa * inv, cp = wp * inv;
    const float4 a = la == -INFINITY ? make_float4(0.f, 0.f, 0.f, 0.f) : o_acc[i];
    const float4 b = o_part[i];
    o_acc[i] = make_float4(a.x * ca + b.x * cp, a.y * ca + b.y * cp, a.z * ca + b.z * cp, a.w * ca + b.w * cp);
    if ((i & 15) == 0) lse_acc[row] = m + logf(wa + wp);
}

__global__ void f32_to_bf16_kernel(const float4* __restrict__ src, uint2* __restrict__ dst, long long n4) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
        const float4 v = src[i];
        __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y);
        __nv_bfloat162 hi = __floats2bfloat162_rn(v.z, v.w);
        uint2 o;
        o.x = *reinterpret_cast<uint32_t*>(&lo);
        o.y = *reinterpret_cast<uint32_t*>(&hi);
        dst[i] = o;
    }
}

__global__ void f32_to_bf16_tail_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, long long start,
                                        long long n) {
    const long long i = start + threadIdx.x;
    if (i < n) dst[i] = __float2bfloat16_rn(src[i]);
}

}  // namespace bfk

extern "C" int blackflash_lse_merge(float* O_acc, float* lse_acc, const float* O_part, const float* lse_part,
                                    long long rows, int d, void* stream) {
    if (d != 64) return bf_set_error(BF_ERR_ARG, "lse_merge supports d=64 only");
    if (rows < 0) return bf_set_error(BF_ERR_ARG, "rows must be >= 0");
    if (rows == 0) return BF_OK;
    if (!O_acc || !lse_acc || !O_part || !lse_part) return bf_set_error(BF_ERR_ARG, "null pointer");
    if (((uintptr_t)O_acc | (uintptr_t)O_part) & 15u) return bf_set_error(BF_ERR_ARG, "O buffers must be 16-byte aligned");
    const long long n4 = rows * 16;
    const int threads = 256;
    const long long blocks = (n4 + threads - 1) / threads;
    if (blocks > 0x7fffffffLL) return bf_set_error(BF_ERR_ARG, "too many rows");
    bfk::lse_merge_kernel<<<(unsigned)blocks, threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<float4*>(O_acc), lse_acc, reinterpret_cast<const float4*>(O_part), lse_part, rows);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return bf_set_error(BF_ERR_CUDA, cudaGetErrorString(e));
    return BF_OK;
}

extern "C" int blackflash_f32_to_bf16(const float* src, void* dst, long long n, void* stream) {
    if (n < 0) return bf_set_error(BF_ERR_ARG, "n must be >= 0");
    if (n == 0) return BF_OK;
    if (!src || !dst) return bf_set_error(BF_ERR_ARG, "null pointer");
    if (((uintptr_t)src & 15u) || ((uintptr_t)dst & 7u)) return bf_set_error(BF_ERR_ARG, "src must be 16-byte and dst 8-byte aligned");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const long long n4 = n / 4;
    if (n4 > 0) {
        long long blocks = (n4 + 255) / 256;
        if (blocks > 148LL * 16) blocks = 148LL * 16;
        bfk::f32_to_bf16_kernel<<<(unsigned)blocks, 256, 0, st>>>(reinterpret_cast<const float4*>(src),
                                                                 reinterpret_cast<uint2*>(dst), n4);
    }
    if (n4 * 4 < n)
        bfk::f32_to_bf16_tail_kernel<<<1, 32, 0, st>>>(src, reinterpret_cast<__nv_bfloat16*>(dst), n4 * 4, n);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return bf_set_error(BF_ERR_CUDA, cudaGetErrorString(e));
    return BF_OK;
}
