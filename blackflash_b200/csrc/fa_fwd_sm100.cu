// BlackFlash-B200: FlashAttention-2 style forward for sm_100a (B200).
//
// Replaces the reference's kernel/flash_attn_mma.cu (flash_attn_naive_kernel,
// :25-465, and its launcher flash_attn_naive_launch, :470-518). Same math:
// O = softmax(scale * Q K^T) V per (b, h), non-causal, bf16 in / bf16 out,
// fp32 accumulation. The reference's row-max / logsumexp slots
// (include/flash_attn.cuh:27-28, never written there) are filled here.
//
// Structure of one CTA (384 threads, one CTA per SM):
//   * two 128-row query tiles of one (b, h) slice -> 256 query rows;
//   * warps 0-3 / 4-7: softmax warpgroups for query tile 0 / 1. One thread
//     owns one query row (= one TMEM lane), so row max / row sum need no
//     shuffles. They also rescale O in TMEM (lazily) and run the epilogue;
//   * warp 8: TMA producer (Q once; K and V per 128-row KV tile into a
//     STAGES-deep mbarrier ring, 128-byte swizzle);
//   * warp 9: allocates TMEM and issues every tcgen05.mma:
//       S_t = Q_t K_j^T   (M=128, N=128, K=64; A,B from smem)      -> TMEM
//       O_t += P_t V_j    (M=128, N=64,  K=128; A=P from TMEM, B=V) -> TMEM
//     P_t is written by the softmax threads as bf16 over the first 64
//     columns of S_t, so P never leaves the SM.
// TMEM columns: S0 [0,128) S1 [128,256) O0 [256,320) O1 [320,384).
//
// MMA issue order per KV tile j: PV0(j-1), S0(j), PV1(j-1), S1(j). Because
// tcgen05 ops from one thread complete in order and the commit that signals
// "S_t(j) ready" is issued after PV_t(j-1), a softmax warpgroup that has
// observed S_t(j) may read/rescale O_t without racing the tensor core.
//
// Every mbarrier wait is bounded (WaitCtl): a lost arrival sets a status
// word and the kernel unwinds instead of spinning forever.
#include "sm100_ptx.cuh"
#include "fa_fwd_sm100.h"

#include <cuda_bf16.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

namespace bfk {

// Set by a bounded wait that gave up; read by blackflash_status().
__device__ unsigned int g_wait_status = 0;

constexpr int kD = 64;          // head dimension
constexpr int kBM = 128;        // query rows per tile
constexpr int kBN = 128;        // KV rows per tile
constexpr int kQTiles = 2;      // query tiles per CTA
constexpr int kStages = 3;      // K/V ring depth
constexpr int kThreads = 384;
constexpr int kTileBytes = kBM * kD * 2;  // 16 KiB (Q, K or V tile, bf16)
constexpr int kTmemCols = 512;

// Shared-memory layout, offsets from a 1024-byte aligned base.
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kQTiles * kTileBytes;
constexpr int kOffV = kOffK + kStages * kTileBytes;
constexpr int kOffBar = kOffV + kStages * kTileBytes;

struct Bars {
    uint64_t q_full;
    uint64_t k_full[kStages];
    uint64_t k_empty[kStages];
    uint64_t v_full[kStages];
    uint64_t v_empty[kStages];
    uint64_t s_full[kQTiles];
    uint64_t p_full[kQTiles];
    uint64_t o_full[kQTiles];
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
};

constexpr int kSmemBytes = kOffBar + (int)sizeof(Bars) + 1024;  // + alignment slack

// Status codes written by a bounded wait that gave up (first one wins).
enum : unsigned {
    kSiteProdKEmpty = 0x101,
    kSiteProdVEmpty = 0x102,
    kSiteMmaQ = 0x201,
    kSiteMmaK = 0x202,
    kSiteMmaV = 0x203,
    kSiteMmaP = 0x204,
    kSiteSoftS = 0x301,
    kSiteSoftO = 0x302,
};

struct KParams {
    int n_q;        // query rows per slice
    int n_kv;       // key/value rows per slice
    int q_blocks;   // ceil(n_q / 256)
    float scale_log2;  // scale * log2(e)
    float scale;
    float* lse;     // [BH, n_q] natural-log logsumexp of scale*S, optional
    float* row_max; // [BH, n_q] max_j scale*S_ij, optional
    float* o_f32;   // [BH, n_q, 64] fp32 normalised output (partial mode), else null
    unsigned long long timeout_ns;
    float* dbg_s;   // optional: raw S of (CTA 0, tile 0, KV tile 0), 128x128 fp32
    int skip_k_loads;  // test hook: producer never loads K (forces a wait timeout)
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

template <bool kF32Out>
__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                        const KParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int bh = blockIdx.x / p.q_blocks;
    const int q_row0 = (blockIdx.x % p.q_blocks) * (kQTiles * kBM);
    const int nk = (p.n_kv + kBN - 1) / kBN;

    if (threadIdx.x == 0) {
        mbar_init(smem_addr(&bars->q_full), 1);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_addr(&bars->k_full[s]), 1);
            mbar_init(smem_addr(&bars->k_empty[s]), 1);
            mbar_init(smem_addr(&bars->v_full[s]), 1);
            mbar_init(smem_addr(&bars->v_empty[s]), 1);
        }
        for (int t = 0; t < kQTiles; ++t) {
            mbar_init(smem_addr(&bars->s_full[t]), 1);
            mbar_init(smem_addr(&bars->p_full[t]), kBM);
            mbar_init(smem_addr(&bars->o_full[t]), 1);
        }
        mbar_init(smem_addr(&bars->drain), 1);
        bars->abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 8 && lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        if (!kF32Out) tma_prefetch_desc(&tmO);
    }
    if (warp == 9) {
        tmem_alloc(smem_addr(&bars->tmem_base), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    const WaitCtl ctl{&bars->abort_flag, &g_wait_status, p.timeout_ns};

    // Launch budget is 168 regs x 384 threads; give the softmax warpgroups
    // 216 each (they hold a 128-column S row) and the TMA/MMA warpgroup 72:
    // 216*256 + 72*128 = 64512 = 168*384.
    if (warp < 8)
        regs_inc<216>();
    else
        regs_dec<72>();

    if (warp < 8) {
        // ------------------------------------------------------------ softmax
        const int t = warp >> 2;                 // query tile of this warpgroup
        const int row = (warp & 3) * 32 + lane;  // row within the tile == TMEM lane
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tS = tmem + lane_off + (uint32_t)(t * kBN);
        const uint32_t tO = tmem + lane_off + (uint32_t)(2 * kBN + t * kD);
        const float sl2 = p.scale_log2;
        const uint32_t bar_s = smem_addr(&bars->s_full[t]);
        const uint32_t bar_p = smem_addr(&bars->p_full[t]);

        float m_use = -INFINITY;  // reference max (log2 domain) the current P/O/l are relative to
        float m_raw = -INFINITY;  // true running max of raw scores
        float l_sum = 0.f;
        bool ok = true;

        for (int j = 0; j < nk; ++j) {
            ok = __all_sync(0xffffffffu, mbar_wait(bar_s, (uint32_t)(j & 1), ctl, kSiteSoftS));
            if (!ok) break;
            tc_fence_after();

            uint32_t s[4][32];
            tmem_ld32(tS + 0, s[0]);
            tmem_ld32(tS + 32, s[1]);
            tmem_ld32(tS + 64, s[2]);
            tmem_ld32(tS + 96, s[3]);
            tmem_wait_ld();

            if (p.dbg_s != nullptr && blockIdx.x == 0 && t == 0 && j == 0) {
#pragma unroll
                for (int c = 0; c < kBN; ++c) p.dbg_s[row * kBN + c] = __uint_as_float(s[c >> 5][c & 31]);
            }

            const int valid = p.n_kv - j * kBN;  // >= 1
            if (valid < kBN) {
#pragma unroll
                for (int c = 0; c < kBN; ++c)
                    if (c >= valid) s[c >> 5][c & 31] = __float_as_uint(-INFINITY);
            }

            float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                mx0 = fmaxf(mx0, __uint_as_float(s[0][c]));
                mx1 = fmaxf(mx1, __uint_as_float(s[1][c]));
                mx2 = fmaxf(mx2, __uint_as_float(s[2][c]));
                mx3 = fmaxf(mx3, __uint_as_float(s[3][c]));
            }
            const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
            m_raw = fmaxf(m_raw, mx);
            const float m_new = mx * sl2;

            // Lazy rescale: keep the old reference max unless the tile max exceeds
            // it by more than 8 (log2 units), i.e. P entries stay <= 256.
            const bool need = m_new > m_use + 8.0f;
            float alpha = 1.f;
            if (need) {
                alpha = fast_exp2(m_use - m_new);  // 0 on the first tile
                m_use = m_new;
            }
            l_sum *= alpha;
            if (j > 0 && __any_sync(0xffffffffu, need)) {
                uint32_t o[32];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    tmem_ld32(tO + h * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
                    tmem_st32(tO + h * 32, o);
                }
            }

            const float neg_m = -m_use;
            float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint32_t pk[16];
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    const float p0 = fast_exp2(fmaf(__uint_as_float(s[q][2 * c]), sl2, neg_m));
                    const float p1 = fast_exp2(fmaf(__uint_as_float(s[q][2 * c + 1]), sl2, neg_m));
                    sum0 += p0;
                    sum1 += p1;
                    pk[c] = pack_bf16x2(p0, p1);
                }
                // bf16 P column q*16.. covers S columns already consumed (32q..32q+31 >= 16q..).
                tmem_st16(tS + q * 16, pk);
            }
            l_sum += sum0 + sum1;
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar_p);
        }

        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(smem_addr(&bars->o_full[t]), 0u, ctl, kSiteSoftO));
        if (ok) {
            tc_fence_after();
            uint32_t o[2][32];
            tmem_ld32(tO, o[0]);
            tmem_ld32(tO + 32, o[1]);
            tmem_wait_ld();
            const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
            const int q_row = q_row0 + t * kBM + row;
            const bool row_ok = q_row < p.n_q;

            if constexpr (kF32Out) {
                if (row_ok) {
                    float4* dst = reinterpret_cast<float4*>(p.o_f32 + ((size_t)bh * p.n_q + q_row) * kD);
#pragma unroll
                    for (int c = 0; c < 16; ++c) {
                        const uint32_t* src = &o[c >> 3][(c & 7) * 4];
                        dst[c] = make_float4(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv,
                                             __uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv);
                    }
                }
            } else {
                // Stage the bf16 tile in this tile's Q buffer (all MMAs reading it are done),
                // in the 128-byte-swizzled image the O tensor map expects, then TMA-store it.
                uint8_t* stage = smem + kOffQ + t * kTileBytes;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const uint32_t* src = &o[c >> 2][(c & 3) * 8];
                    uint4 v;
                    v.x = pack_bf16x2(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv);
                    v.y = pack_bf16x2(__uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv);
                    v.z = pack_bf16x2(__uint_as_float(src[4]) * inv, __uint_as_float(src[5]) * inv);
                    v.w = pack_bf16x2(__uint_as_float(src[6]) * inv, __uint_as_float(src[7]) * inv);
                    *reinterpret_cast<uint4*>(stage + row * 128 + ((c ^ (row & 7)) << 4)) = v;
                }
                fence_proxy_async_smem();
                named_bar_sync(1 + t, 128);
                if ((warp & 3) == 0 && lane == 0) {
                    tma_store_3d(&tmO, smem_addr(stage), 0, q_row0 + t * kBM, bh);
                    tma_store_commit();
                    tma_store_wait_read0();
                }
            }
            if (row_ok) {
                const size_t idx = (size_t)bh * p.n_q + q_row;
                if (p.lse) p.lse[idx] = (m_use + __log2f(l_sum)) * 0.69314718055994531f;
                if (p.row_max) p.row_max[idx] = m_raw * p.scale;
            }
        }
    } else if (warp == 8) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            const uint32_t q_full = smem_addr(&bars->q_full);
            mbar_arrive_expect_tx(q_full, kQTiles * kTileBytes);
            for (int t = 0; t < kQTiles; ++t)
                tma_load_3d(smem_addr(smem + kOffQ + t * kTileBytes), &tmQ, q_full, 0, q_row0 + t * kBM, bh);
            int last_k = -1, last_v = -1;
            for (int j = 0; j < nk; ++j) {
                const int st = j % kStages;
                const uint32_t par = ((uint32_t)(j / kStages) & 1u) ^ 1u;
                if (!mbar_wait(smem_addr(&bars->k_empty[st]), par, ctl, kSiteProdKEmpty)) break;
                if (!p.skip_k_loads) {
                    mbar_arrive_expect_tx(smem_addr(&bars->k_full[st]), kTileBytes);
                    tma_load_3d(smem_addr(smem + kOffK + st * kTileBytes), &tmK, smem_addr(&bars->k_full[st]), 0,
                                j * kBN, bh);
                    last_k = j;
                }
                if (!mbar_wait(smem_addr(&bars->v_empty[st]), par, ctl, kSiteProdVEmpty)) break;
                mbar_arrive_expect_tx(smem_addr(&bars->v_full[st]), kTileBytes);
                tma_load_3d(smem_addr(smem + kOffV + st * kTileBytes), &tmV, smem_addr(&bars->v_full[st]), 0,
                            j * kBN, bh);
                last_v = j;
            }
            if (*ctl.abort_flag) {
                // Let copies still in flight land before the CTA's shared memory is released.
                int never = 0;
                const WaitCtl drain{&never, nullptr, ctl.limit_ns};
                if (last_k >= 0)
                    mbar_wait(smem_addr(&bars->k_full[last_k % kStages]), (uint32_t)(last_k / kStages) & 1u, drain, 0);
                if (last_v >= 0)
                    mbar_wait(smem_addr(&bars->v_full[last_v % kStages]), (uint32_t)(last_v / kStages) & 1u, drain, 0);
                mbar_wait(smem_addr(&bars->q_full), 0u, drain, 0);
            }
        }
    } else if (warp == 9) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t kIdescS = idesc_bf16_f32(kBM, kBN, 0);  // Q (K-major) x K (K-major)
            constexpr uint32_t kIdescO = idesc_bf16_f32(kBM, kD, 1);   // P (TMEM)   x V (MN-major)
            const uint32_t tS0 = tmem;
            const uint32_t tO0 = tmem + 2 * kBN;

            bool ok = mbar_wait(smem_addr(&bars->q_full), 0u, ctl, kSiteMmaQ);
            tc_fence_after();

            auto issue_pv = [&](int t, int vst, bool acc) {
                const uint64_t v_desc = smem_desc_sw128(smem_addr(smem + kOffV + vst * kTileBytes), 16, 1024);
#pragma unroll
                for (int kk = 0; kk < kBN / 16; ++kk) {
                    // K step of 16 KV rows: 8 TMEM columns of packed bf16 P, 16 rows x 128 B of V.
                    umma_ts(tO0 + t * kD, tS0 + t * kBN + kk * 8, v_desc + (uint64_t)((kk * 16 * 128) >> 4), kIdescO,
                            (acc || kk > 0) ? 1u : 0u);
                }
            };
            auto issue_s = [&](int t, int kst) {
                const uint64_t k_desc = smem_desc_sw128(smem_addr(smem + kOffK + kst * kTileBytes), 16, 1024);
                const uint64_t q_desc = smem_desc_sw128(smem_addr(smem + kOffQ + t * kTileBytes), 16, 1024);
#pragma unroll
                for (int kk = 0; kk < kD / 16; ++kk) {
                    // K step of 16 head-dim elements = 32 bytes inside the 128-byte swizzle atom.
                    umma_ss(tS0 + t * kBN, q_desc + (uint64_t)((kk * 32) >> 4), k_desc + (uint64_t)((kk * 32) >> 4),
                            kIdescS, kk > 0 ? 1u : 0u);
                }
            };

            for (int j = 0; j < nk && ok; ++j) {
                const int st = j % kStages;
                if (!(ok = mbar_wait(smem_addr(&bars->k_full[st]), (uint32_t)(j / kStages) & 1u, ctl, kSiteMmaK)))
                    break;
                tc_fence_after();
                const int pst = (j + kStages - 1) % kStages;
                for (int t = 0; t < kQTiles && ok; ++t) {
                    if (j > 0) {
                        if (t == 0 && !(ok = mbar_wait(smem_addr(&bars->v_full[pst]), (uint32_t)((j - 1) / kStages) & 1u,
                                                       ctl, kSiteMmaV)))
                            break;
                        if (!(ok = mbar_wait(smem_addr(&bars->p_full[t]), (uint32_t)((j - 1) & 1), ctl, kSiteMmaP)))
                            break;
                        tc_fence_after();
                        issue_pv(t, pst, j - 1 > 0);
                        if (t == kQTiles - 1) umma_commit(smem_addr(&bars->v_empty[pst]));
                    }
                    issue_s(t, st);
                    umma_commit(smem_addr(&bars->s_full[t]));
                }
                if (ok) umma_commit(smem_addr(&bars->k_empty[st]));
            }
            if (ok) {
                const int pst = (nk - 1) % kStages;
                ok = mbar_wait(smem_addr(&bars->v_full[pst]), (uint32_t)((nk - 1) / kStages) & 1u, ctl, kSiteMmaV);
                for (int t = 0; t < kQTiles && ok; ++t) {
                    if (!(ok = mbar_wait(smem_addr(&bars->p_full[t]), (uint32_t)((nk - 1) & 1), ctl, kSiteMmaP))) break;
                    tc_fence_after();
                    issue_pv(t, pst, nk - 1 > 0);
                    umma_commit(smem_addr(&bars->o_full[t]));
                }
                if (ok) umma_commit(smem_addr(&bars->v_empty[pst]));
            }
            // Drain: every MMA issued above has finished before TMEM is released.
            umma_commit(smem_addr(&bars->drain));
            int never = 0;
            WaitCtl drain{&never, nullptr, ctl.limit_ns};
            mbar_wait(smem_addr(&bars->drain), 0u, drain, 0);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace bfk

// ============================================================================ host side
namespace {

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PFN_encodeTiled get_encode_fn() {
    static PFN_encodeTiled fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult qres;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qres) == cudaSuccess &&
            qres == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_encodeTiled>(ptr);
    }
    return fn;
}

// [BH][rows][64] bf16 viewed as a 3-D tensor; 64 x 128-row boxes with 128-byte
// swizzle. Rows past `rows` inside a slice load as zero and are never stored.
int make_map(CUtensorMap* m, const void* base, long long bh, int rows) {
    PFN_encodeTiled enc = get_encode_fn();
    if (!enc) return bf_set_error(BF_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[3] = {(cuuint64_t)bfk::kD, (cuuint64_t)rows, (cuuint64_t)bh};
    cuuint64_t strides[2] = {(cuuint64_t)bfk::kD * 2, (cuuint64_t)rows * bfk::kD * 2};
    cuuint32_t box[3] = {(cuuint32_t)bfk::kD, (cuuint32_t)bfk::kBM, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return bf_set_error(BF_ERR_CUDA, "cuTensorMapEncodeTiled rejected the tensor");
    return BF_OK;
}

template <bool kF32Out>
int configure_once() {
    static bool done[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return bf_set_error(BF_ERR_CUDA, "cudaGetDevice failed");
    if (!done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(bfk::fa_fwd_sm100_kernel<kF32Out>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, bfk::kSmemBytes);
        if (e != cudaSuccess) return bf_set_error(BF_ERR_CUDA, cudaGetErrorString(e));
        done[dev] = true;
    }
    return BF_OK;
}

}  // namespace

int bf_fwd_launch(const BfFwdArgs* a) {
    if (a->d != bfk::kD) return bf_set_error(BF_ERR_ARG, "BlackFlash currently only supports d=64");
    if (a->bh <= 0 || a->n_q <= 0 || a->n_kv <= 0) return bf_set_error(BF_ERR_ARG, "empty problem: B*H and N must be >= 1");
    if (!a->q || !a->k || !a->v || (!a->o && !a->o_f32)) return bf_set_error(BF_ERR_ARG, "null tensor pointer");
    auto misaligned = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) != 0; };
    if (misaligned(a->q) || misaligned(a->k) || misaligned(a->v) || (a->o && misaligned(a->o)) ||
        (a->o_f32 && misaligned(a->o_f32)))
        return bf_set_error(BF_ERR_ARG, "Q/K/V/O must be 16-byte aligned");
    const long long q_blocks = (a->n_q + bfk::kQTiles * bfk::kBM - 1) / (bfk::kQTiles * bfk::kBM);
    const long long grid = q_blocks * a->bh;
    if (grid > 0x7fffffffLL || a->bh > 0x7fffffffLL) return bf_set_error(BF_ERR_ARG, "problem too large for one launch");

    CUtensorMap mq, mk, mv, mo;
    int rc;
    if ((rc = make_map(&mq, a->q, a->bh, a->n_q)) != BF_OK) return rc;
    if ((rc = make_map(&mk, a->k, a->bh, a->n_kv)) != BF_OK) return rc;
    if ((rc = make_map(&mv, a->v, a->bh, a->n_kv)) != BF_OK) return rc;
    if (a->o) {
        if ((rc = make_map(&mo, a->o, a->bh, a->n_q)) != BF_OK) return rc;
    } else {
        mo = mq;  // not read in fp32-output mode
    }

    bfk::KParams kp;
    kp.n_q = a->n_q;
    kp.n_kv = a->n_kv;
    kp.q_blocks = (int)q_blocks;
    kp.scale = a->scale;
    kp.scale_log2 = a->scale * 1.4426950408889634f;
    kp.lse = a->lse;
    kp.row_max = a->row_max;
    kp.o_f32 = a->o_f32;
    kp.timeout_ns = a->timeout_ns ? a->timeout_ns : 4000000000ull;
    kp.dbg_s = a->dbg_s;
    kp.skip_k_loads = a->skip_k_loads;

    cudaStream_t stream = reinterpret_cast<cudaStream_t>(a->stream);
    if (a->o_f32) {
        if ((rc = configure_once<true>()) != BF_OK) return rc;
        bfk::fa_fwd_sm100_kernel<true><<<(unsigned)grid, bfk::kThreads, bfk::kSmemBytes, stream>>>(mq, mk, mv, mo, kp);
    } else {
        if ((rc = configure_once<false>()) != BF_OK) return rc;
        bfk::fa_fwd_sm100_kernel<false><<<(unsigned)grid, bfk::kThreads, bfk::kSmemBytes, stream>>>(mq, mk, mv, mo, kp);
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return bf_set_error(BF_ERR_CUDA, cudaGetErrorString(e));
    return BF_OK;
}

extern "C" int blackflash_status(int reset, unsigned* out) {
    unsigned v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, bfk::g_wait_status, sizeof(v));
    if (e != cudaSuccess) return bf_set_error(BF_ERR_CUDA, cudaGetErrorString(e));
    if (reset) {
        const unsigned zero = 0;
        e = cudaMemcpyToSymbol(bfk::g_wait_status, &zero, sizeof(zero));
        if (e != cudaSuccess) return bf_set_error(BF_ERR_CUDA, cudaGetErrorString(e));
    }
    if (out) *out = v;
    return BF_OK;
}
