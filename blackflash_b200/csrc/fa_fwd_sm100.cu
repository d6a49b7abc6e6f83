// BlackFlash-B200: FlashAttention-2 style forward for sm_100a (B200).
//
// Replaces the reference's kernel/flash_attn_mma.cu (flash_attn_naive_kernel,
// :25-465, and its launcher flash_attn_naive_launch, :470-518). Same math:
// O = softmax(scale * Q K^T) V per (b, h), non-causal, bf16 in / bf16 out,
// fp32 accumulation. The reference's row-max / logsumexp slots
// (include/flash_attn.cuh:27-28, never written there) are filled here.
//
// Persistent kernel: one CTA per SM (640 threads) walks work items
// item = blockIdx.x + k * gridDim.x; an item is two 128-row query tiles
// (256 rows) of one (b, h) slice against all of its KV rows. Roles:
//   * warps 0-7 / 8-15: softmax for query tile 0 / 1, four warps per
//     scheduler. Each warp covers 16 rows (TMEM lanes); two threads of the
//     warp share a row, one per 64-column half of S (tcgen05 16x32bx2
//     shapes), so the row max takes one shuffle. They also rescale O in TMEM
//     (lazily) and run the epilogue;
//   * warp 16: TMA producer: Q (double-buffered across items) and K / V per
//     128-row KV tile into a kStages-deep mbarrier ring, 128-byte swizzle;
//   * warps 17 / 18: issue the tcgen05.mma streams (S / PV), warp 17 owns TMEM:
//       S_t = Q_t K_j^T   (M=128, N=128, K=64; A,B from smem)      -> TMEM
//       O_t += P_t V_j    (M=128, N=64,  K=128; A=P from TMEM, B=V) -> TMEM
//     P_t is written by the softmax threads as bf16 into its own TMEM
//     columns, so P never leaves the SM.
// TMEM columns (all 512): S0 [0,128) S1 [128,256) P0 [256,320) P1 [320,384)
//                         O0 [384,448) O1 [448,512).
//
// Pipelining. Each MMA issuer walks one flat stream of KV steps across work
// items (S(g) for both tiles; PV(g) for both tiles). A softmax
// warpgroup releases S_t (s_empty) as soon as S_t(g) is in registers, so the
// tensor core computes S_t(g+1) - possibly the next item's - while the
// exponentials of step g run; it waits for PV_t(g-1) (pv_done) only before it
// overwrites P_t or touches O_t. The next item's Q / K / V are in flight
// while the current item's last steps and epilogue run.
//
// Exponentials: p = 2^(s * scale * log2 e - m). Most run on MUFU (ex2); a fixed
// share (kEmuPairs of every kEmuPeriod pairs) runs on the FMA pipe (exp2_poly_x2) so both
// pipes share the load. Arithmetic on pairs uses the sm_100 f32x2 forms.
//
// Every mbarrier wait is bounded (WaitCtl): a lost arrival sets a status
// word and the kernel unwinds instead of spinning forever.
#include "sm100_ptx.cuh"
#include "fa_fwd_sm100.h"

#include <cuda_bf16.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <utility>

namespace bfk {

// Set by a bounded wait that gave up; read by blackflash_status().
__device__ unsigned int g_wait_status = 0;

constexpr int kD = 64;          // head dimension
constexpr int kBM = 128;        // query rows per tile
constexpr int kBN = 128;        // KV rows per tile
constexpr int kQTiles = 2;      // query tiles per work item
#ifndef BF_KV_STAGES
#define BF_KV_STAGES 3
#endif
constexpr int kStages = BF_KV_STAGES;  // K/V ring depth
constexpr int kSoftWarps = 16;                       // 8 per query tile, 4 per scheduler
#ifndef BF_REGSPLIT
#define BF_REGSPLIT 1
#endif
// With BF_REGSPLIT the block is 20 warps (a fourth, idle warp completes the last
// warpgroup) so setmaxnreg can move registers from the issuer warps to the softmax.
constexpr int kThreads = kSoftWarps * 32 + (BF_REGSPLIT ? 4 : 3) * 32;  // + TMA producer, S issuer, PV issuer
#ifndef BF_SOFT_REGS
#define BF_SOFT_REGS 104
#endif
constexpr int kSoftRegs = BF_SOFT_REGS, kIssueRegs = (96 * 640 - BF_SOFT_REGS * 512) / 128 / 8 * 8;
constexpr int kTileBytes = kBM * kD * 2;  // 16 KiB (Q, K, V or O tile, bf16)
constexpr int kTmemCols = 512;
// TMEM columns: S_t at t*128; P_t (bf16, 64 columns) and O_t (fp32, 64 columns) after them.
constexpr int kColS = 0;
constexpr int kColP = 2 * 128;
constexpr int kColO = kColP + 2 * 64;
static_assert(kColO + 2 * 64 <= kTmemCols, "TMEM columns");
constexpr int kProducerWarp = 16;  // TMA producer
constexpr int kSWarp = 17;         // issues S = Q K^T; owns the TMEM allocation
constexpr int kPVWarp = 18;        // issues O += P V
#ifndef BF_EMU_PAIRS
#define BF_EMU_PAIRS 1
#endif
#ifndef BF_EMU_PERIOD
#define BF_EMU_PERIOD 8
#endif
constexpr int kEmuPairs = BF_EMU_PAIRS;    // of every kEmuPeriod exp2 pairs, how many run on the FMA pipe
constexpr int kEmuPeriod = BF_EMU_PERIOD;  // 8, 16 or 32 (a thread holds 32 pairs per step)
static_assert(kEmuPeriod == 8 || kEmuPeriod == 16 || kEmuPeriod == 32, "kEmuPeriod must divide 32");

// Shared-memory layout, offsets from a 1024-byte aligned base.
constexpr int kOffQ = 0;                                  // [2 buffers][2 tiles]
constexpr int kOffK = kOffQ + 2 * kQTiles * kTileBytes;   // [kStages]
constexpr int kOffV = kOffK + kStages * kTileBytes;       // [kStages]
constexpr int kOffO = kOffV + kStages * kTileBytes;       // [2 tiles] bf16 output staging
constexpr int kOffBar = kOffO + kQTiles * kTileBytes;

struct Bars {
    uint64_t q_full[2];
    uint64_t q_empty[2];
    uint64_t k_full[kStages];
    uint64_t k_empty[kStages];
    uint64_t v_full[kStages];
    uint64_t v_empty[kStages];
    uint64_t s_full[kQTiles];
    uint64_t s_empty[kQTiles];
    uint64_t p_full[kQTiles];
    uint64_t pv_done[kQTiles];
    uint64_t drain;
    uint64_t drain_pv;
    uint32_t tmem_base;
    int abort_flag;
};

constexpr int kSmemBytes = kOffBar + (int)sizeof(Bars) + 1024;  // + alignment slack

// Status codes written by a bounded wait that gave up (first one wins).
enum : unsigned {
    kSiteProdQEmpty = 0x100,
    kSiteProdKEmpty = 0x101,
    kSiteProdVEmpty = 0x102,
    kSiteMmaQ = 0x201,
    kSiteMmaK = 0x210,  // +0 K full, +1 S_0 empty, +2 S_1 empty
    kSiteMmaV = 0x220,  // +0 V full, +1 P_0 full, +2 P_1 full
    kSiteSoftS = 0x301,
    kSiteSoftO = 0x302,
    kSiteSoftPV = 0x303,
};

struct KParams {
    int n_q;        // query rows per slice
    int n_kv;       // key/value rows per slice
    int q_blocks;   // ceil(n_q / 256)
    int items;      // bh * q_blocks
    float scale_log2;  // scale * log2(e)
    float scale;
    float* lse;     // [BH, n_q] natural-log logsumexp of scale*S, optional
    float* row_max; // [BH, n_q] max_j scale*S_ij, optional
    float* o_f32;   // [BH, n_q, 64] fp32 normalised output (partial mode), else null
    unsigned long long timeout_ns;
    float* dbg_s;   // optional: raw S of (item 0, tile 0, KV tile 0), 128x128 fp32
    int skip_k_loads;  // test hook: producer never loads K (forces a wait timeout)
    int causal;        // key j visible to query i only if j <= i (top-left aligned)
    long long* trace;  // kTrace builds: clock64 event stamps of CTA `trace_cta`
    int trace_cta;
    // Blocked KV: K/V maps cover [kv_blocks * bh] slices of kv_blk_tiles * 128 rows; KV tile j
    // of slice bh lives in block j / kv_blk_tiles (past kv_skip) at slice block * bh_count + bh.
    int kv_blk_tiles;  // 0: plain layout
    int kv_skip;       // block left out, -1 for none
    int bh_count;
};

// KV tile j of slice bh -> (row, slice) coordinates in the K/V tensor maps.
__device__ __forceinline__ void kv_coords(const KParams& p, int j, int bh, int& row, int& slice) {
    if (p.kv_blk_tiles == 0) {
        row = j * kBN;
        slice = bh;
        return;
    }
    int blk = j / p.kv_blk_tiles;
    if (p.kv_skip >= 0 && blk >= p.kv_skip) ++blk;
    row = (j - (j / p.kv_blk_tiles) * p.kv_blk_tiles) * kBN;
    slice = blk * p.bh_count + bh;
}

// Pipeline event trace (diagnostic builds only): trace[role * 512 + g * 8 + ev]
// holds clock64() - t0 of CTA p.trace_cta for its first 64 global KV steps.
// Roles: 0/1 softmax warpgroup 0/1 (lane 0 of its first warp), 2 MMA issuer,
// 3 TMA producer.
#define BF_TRACE(role, g, ev)                                                                       \
    do {                                                                                            \
        if constexpr (kTrace) {                                                                     \
            if (tracing && (g) < 64) p.trace[(role) * 512 + (g) * 8 + (ev)] = clock64() - trace_t0; \
        }                                                                                           \
    } while (0)

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Work item -> (slice, first query row). With the causal mask the late query
// blocks carry the most KV tiles, so they are handed out first.
__device__ __forceinline__ void decode_item(const KParams& p, int item, int& bh, int& q_row0) {
    bh = item / p.q_blocks;
    int qb = item % p.q_blocks;
    if (p.causal) qb = p.q_blocks - 1 - qb;
    q_row0 = qb * (kQTiles * kBM);
}

// KV tiles an item visits: all of them, or with the causal mask those up to the
// item's last query row (the diagonal tiles are masked element-wise).
__device__ __forceinline__ int item_kv_tiles(const KParams& p, int q_row0, int nk) {
    if (!p.causal) return nk;
    const int last_row = min(q_row0 + kQTiles * kBM, p.n_q) - 1;
    return min(last_row / kBN + 1, nk);
}

template <bool kF32Out, bool kTrace = false>
__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                        const KParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nk = (p.n_kv + kBN - 1) / kBN;
    const long long trace_t0 = kTrace ? clock64() : 0;
    const bool trace_hit = kTrace && (int)blockIdx.x == p.trace_cta;
    // Trace builds also record, for every CTA, the global timer (ns) at entry, after the
    // set-up, when its first S tile is ready and at exit: trace[4 * 512 + cta * 4 + k].
    if constexpr (kTrace) {
        if (threadIdx.x == 0) p.trace[4 * 512 + blockIdx.x * 4 + 0] = (long long)global_timer_ns();
    }

    if (threadIdx.x == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_addr(&bars->q_full[b]), 1);
            mbar_init(smem_addr(&bars->q_empty[b]), 1);
        }
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_addr(&bars->k_full[s]), 1);
            mbar_init(smem_addr(&bars->k_empty[s]), 1);
            mbar_init(smem_addr(&bars->v_full[s]), 1);
            mbar_init(smem_addr(&bars->v_empty[s]), 1);
        }
        for (int t = 0; t < kQTiles; ++t) {
            mbar_init(smem_addr(&bars->s_full[t]), 1);
            mbar_init(smem_addr(&bars->s_empty[t]), 8);  // one arrival per softmax warp of the tile
            mbar_init(smem_addr(&bars->p_full[t]), 8);
            mbar_init(smem_addr(&bars->pv_done[t]), 1);
        }
        mbar_init(smem_addr(&bars->drain), 1);
        mbar_init(smem_addr(&bars->drain_pv), 1);
        bars->abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == kProducerWarp && lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        if (!kF32Out) tma_prefetch_desc(&tmO);
    }
    if (warp == kSWarp) {
        tmem_alloc(smem_addr(&bars->tmem_base), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    const WaitCtl ctl{&bars->abort_flag, &g_wait_status, p.timeout_ns};
    // The set-up above (barriers, TMEM, descriptor prefetch) touches no global data, so
    // with programmatic dependent launch it overlaps the previous grid's tail; every
    // global read or write comes after the wait. The next grid may be scheduled as soon
    // as this one's CTAs start to exit.
    griddep_launch_dependents();
    griddep_wait();
    if constexpr (kTrace) {
        if (threadIdx.x == 0) p.trace[4 * 512 + blockIdx.x * 4 + 1] = (long long)global_timer_ns();
    }

#if BF_REGSPLIT
    // Launch budget 96 x 640 = 61440 registers: softmax kSoftRegs x 512 + issuers kIssueRegs x 128.
    static_assert(kSoftRegs * kSoftWarps * 32 + kIssueRegs * (kThreads - kSoftWarps * 32) <= 96 * kThreads,
                  "register split exceeds the launch budget");
    if (warp < kSoftWarps)
        regs_inc<kSoftRegs>();
    else
        regs_dec<kIssueRegs>();
#endif
    if (warp < kSoftWarps) {
        // ------------------------------------------------------------ softmax
        // Tile t has 8 warps. Warp w covers 16 TMEM lanes (rows) of its lane
        // quarter (w % 4); within the warp, lanes i and i + 16 share a row,
        // lane i < 16 holding S columns [0, 64) and lane i + 16 columns [64, 128)
        // (tcgen05 16x32bx2 shapes). The row max needs one shuffle; the row
        // sum stays per half and is combined in the epilogue.
        const int t = warp >> 3;
        const int quarter = warp & 3;
        const int sub = (warp >> 2) & 1;
        const int h = lane >> 4;  // column half
        const int row = quarter * 32 + sub * 16 + (lane & 15);  // row within the tile == TMEM lane
        const uint32_t lane_off = (uint32_t)(quarter * 32 + sub * 16) << 16;
        const uint32_t tS = tmem + lane_off + (uint32_t)(kColS + t * kBN);
        const uint32_t tP = tmem + lane_off + (uint32_t)(kColP + t * kD);
        const uint32_t tO = tmem + lane_off + (uint32_t)(kColO + t * kD);
        const float sl2 = p.scale_log2;
        const uint64_t sl2_2 = f2_pack(sl2, sl2);
        const uint32_t bar_s = smem_addr(&bars->s_full[t]);
        const uint32_t bar_se = smem_addr(&bars->s_empty[t]);
        const uint32_t bar_p = smem_addr(&bars->p_full[t]);
        const uint32_t bar_pv = smem_addr(&bars->pv_done[t]);
        // P_t is rewritten only after PV_t of the previous step has read it.
        const uint32_t bar_preuse = bar_pv;
        const bool issuer = (warp & 7) == 0 && lane == 0;  // issues tile t's TMA stores
        const bool tracing = trace_hit && issuer;
        uint8_t* stage = smem + kOffO + t * kTileBytes;
        uint32_t g = 0;  // global KV step of this CTA
        bool ok = true;

        for (int item = blockIdx.x; item < p.items && ok; item += gridDim.x) {
            int bh, q_row0;
            decode_item(p, item, bh, q_row0);
            const int nk_item = item_kv_tiles(p, q_row0, nk);
            float m_use = -INFINITY;  // reference max (log2 domain) the current P/O/l are relative to
            float m_raw = -INFINITY;  // true running max of raw scores
            float l_half = 0.f;       // row sum over this thread's column half

            for (int j = 0; j < nk_item; ++j, ++g) {
                BF_TRACE(t, g, 0);
                if (!(ok = warp_wait(bar_s, g & 1u, ctl, kSiteSoftS))) break;
                tc_fence_after();
                BF_TRACE(t, g, 1);
                if constexpr (kTrace) {
                    if (g == 0 && threadIdx.x == 0) p.trace[4 * 512 + blockIdx.x * 4 + 2] = (long long)global_timer_ns();
                }

                uint32_t s[2][32];  // columns 64h + [0, 32) and 64h + [32, 64)
                tmem_ld16x32bx2_x32<64>(tS + 0, s[0]);
                tmem_ld16x32bx2_x32<64>(tS + 32, s[1]);
                tmem_wait_ld();
                BF_TRACE(t, g, 2);

                if (p.dbg_s != nullptr && item == 0 && t == 0 && j == 0) {
#pragma unroll
                    for (int c = 0; c < 64; ++c) p.dbg_s[row * kBN + h * 64 + c] = __uint_as_float(s[c >> 5][c & 31]);
                }

                // Visible keys of this row, relative to this thread's first column
                // (may be <= 0: ragged last tile or, with the causal mask, past the diagonal).
                const int q_abs = q_row0 + t * kBM + row;
                const int kv_lim = p.causal ? min(p.n_kv, q_abs + 1) : p.n_kv;
                const int valid = kv_lim - j * kBN - h * 64;
                if (valid < 64) {
#pragma unroll
                    for (int c = 0; c < 64; ++c)
                        if (c >= valid) s[c >> 5][c & 31] = __float_as_uint(-INFINITY);
                }

                // p = 2^(s * scale * log2 e - m): the argument is one packed FMA per pair;
                // kEmuPairs of every kEmuPeriod pairs take the FMA-pipe exp2, the rest MUFU ex2.
                // Returns this thread's partial row sum; fills pk with bf16 pairs.
                uint32_t pk[2][16];
                auto exps = [&](float m_ref) -> float {
                    const uint64_t negm_2 = f2_pack(-m_ref, -m_ref);
                    uint64_t sum_a = f2_pack(0.f, 0.f), sum_b = f2_pack(0.f, 0.f);
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
#pragma unroll
                        for (int c = 0; c < 16; ++c) {
                            const uint64_t x2 = f2_fma(
                                f2_pack(__uint_as_float(s[q][2 * c]), __uint_as_float(s[q][2 * c + 1])), sl2_2, negm_2);
                            uint64_t p2;
                            if (((q * 16 + c) & (kEmuPeriod - 1)) < kEmuPairs) {
                                p2 = exp2_poly_x2(x2);
                            } else {
                                float x0, x1;
                                f2_unpack(x2, x0, x1);
                                p2 = f2_pack(fast_exp2(x0), fast_exp2(x1));
                            }
                            if (c & 1)
                                sum_b = f2_add(sum_b, p2);
                            else
                                sum_a = f2_add(sum_a, p2);
                            float p0, p1;
                            f2_unpack(p2, p0, p1);
                            pk[q][c] = pack_bf16x2(p0, p1);
                        }
                    }
                    float a0, a1, b0, b1;
                    f2_unpack(sum_a, a0, a1);
                    f2_unpack(sum_b, b0, b1);
                    return (a0 + a1) + (b0 + b1);
                };
                auto row_max = [&]() -> float {
                    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
                    for (int c = 0; c < 32; c += 2) {
                        mx0 = fmax3(mx0, __uint_as_float(s[0][c]), __uint_as_float(s[0][c + 1]));
                        mx1 = fmax3(mx1, __uint_as_float(s[1][c]), __uint_as_float(s[1][c + 1]));
                    }
                    const float mx = fmaxf(mx0, mx1);
                    return fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));  // the row's other half
                };

                // S_t is in registers (tcgen05.wait::ld is warp-wide): one lane tells the
                // S issuer that it may be overwritten.
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar_se);
                const float mx = row_max();
                m_raw = fmaxf(m_raw, mx);
                const float m_new = mx * sl2;
                BF_TRACE(t, g, 3);
                // Lazy rescale: keep the old reference max unless the tile max exceeds
                // it by more than 8 (log2 units), i.e. P entries stay <= 256.
                const bool need = m_new > m_use + 8.0f;
                float alpha = 1.f;
                if (need) {
                    alpha = fast_exp2(m_use - m_new);  // 0 on the first tile
                    m_use = m_new;
                }
                l_half = l_half * alpha + exps(m_use);
                BF_TRACE(t, g, 4);

                // P_t of the previous step must have been consumed (and O_t be final)
                // before we overwrite P_t / rescale O_t.
                if (g > 0) {
                    if (!(ok = warp_wait(bar_preuse, (g - 1) & 1u, ctl, kSiteSoftPV))) break;
                    tc_fence_after();
                }
                BF_TRACE(t, g, 5);
                if (j > 0 && __any_sync(0xffffffffu, need)) {
                    uint32_t o[32];  // O columns 32h + [0, 32)
                    tmem_ld16x32bx2_x32<32>(tO, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
                    tmem_st16x32bx2_x32<32>(tO, o);
                }
                // bf16 P: this thread's 64 S columns are P columns 32h + [0, 32).
                tmem_st16x32bx2_x16<32>(tP, pk[0]);
                tmem_st16x32bx2_x16<32>(tP + 16, pk[1]);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar_p);
                BF_TRACE(t, g, 6);
            }
            if (!ok) break;

            // ---------------------------------------------------- epilogue of this item
            if (!(ok = warp_wait(bar_pv, (g - 1) & 1u, ctl, kSiteSoftO))) break;
            tc_fence_after();
            uint32_t o[32];
            tmem_ld16x32bx2_x32<32>(tO, o);
            tmem_wait_ld();
            const float l_sum = l_half + __shfl_xor_sync(0xffffffffu, l_half, 16);
            const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
            const int q_row = q_row0 + t * kBM + row;
            const bool row_ok = q_row < p.n_q;

            if constexpr (kF32Out) {
                if (row_ok) {
                    float4* dst = reinterpret_cast<float4*>(p.o_f32 + ((size_t)bh * p.n_q + q_row) * kD + h * 32);
#pragma unroll
                    for (int c = 0; c < 8; ++c)
                        dst[c] = make_float4(__uint_as_float(o[4 * c]) * inv, __uint_as_float(o[4 * c + 1]) * inv,
                                             __uint_as_float(o[4 * c + 2]) * inv, __uint_as_float(o[4 * c + 3]) * inv);
                }
            } else {
                // bf16 tile in the 128-byte-swizzled image the O tensor map expects, then TMA store.
                if (issuer) tma_store_wait_read0();  // the previous item's store has left the staging buffer
                named_bar_sync(1 + t, 2 * kBM);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint32_t* src = &o[c * 8];
                    uint4 v;
                    v.x = pack_bf16x2(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv);
                    v.y = pack_bf16x2(__uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv);
                    v.z = pack_bf16x2(__uint_as_float(src[4]) * inv, __uint_as_float(src[5]) * inv);
                    v.w = pack_bf16x2(__uint_as_float(src[6]) * inv, __uint_as_float(src[7]) * inv);
                    const int chunk = h * 4 + c;
                    *reinterpret_cast<uint4*>(stage + row * 128 + ((chunk ^ (row & 7)) << 4)) = v;
                }
                fence_proxy_async_smem();
                named_bar_sync(1 + t, 2 * kBM);
                if (issuer) {
                    tma_store_3d(&tmO, smem_addr(stage), 0, q_row0 + t * kBM, bh);
                    tma_store_commit();
                }
            }
            if (row_ok && h == 0) {
                const size_t idx = (size_t)bh * p.n_q + q_row;
                if (p.lse) p.lse[idx] = (m_use + __log2f(l_sum)) * 0.69314718055994531f;
                if (p.row_max) p.row_max[idx] = m_raw * p.scale;
            }
            BF_TRACE(t, 63, 7);
        }
        if (!kF32Out && issuer) tma_store_wait0();
    } else if (warp == kProducerWarp) {
        // ------------------------------------------------------------ TMA producer
        // The whole warp runs the loop (warp-uniform control flow and
        // addresses); one elected lane issues the copies.
        const bool leader = elect_one();
        const bool tracing = trace_hit && leader;
        const uint32_t q_smem0 = smem_addr(smem + kOffQ);
        const uint32_t k_smem0 = smem_addr(smem + kOffK), v_smem0 = smem_addr(smem + kOffV);
        const uint32_t q_full0 = smem_addr(&bars->q_full[0]), q_empty0 = smem_addr(&bars->q_empty[0]);
        const uint32_t k_full0 = smem_addr(&bars->k_full[0]), k_empty0 = smem_addr(&bars->k_empty[0]);
        const uint32_t v_full0 = smem_addr(&bars->v_full[0]), v_empty0 = smem_addr(&bars->v_empty[0]);
        int last_k = -1, last_v = -1, last_q = -1;  // for the abort drain
        uint32_t c = 0;  // KV tiles issued by this CTA
        int st = 0;
        uint32_t par = 1u;  // parity of the "empty" phase to wait for (fresh barriers pass parity 1)
        bool ok = true;
        int it = 0;
        for (int item = blockIdx.x; item < p.items && ok; item += gridDim.x, ++it) {
            int bh, q_row0;
            decode_item(p, item, bh, q_row0);
            const int nk_item = item_kv_tiles(p, q_row0, nk);
            const int qb = it & 1;
            if (!(ok = warp_wait(q_empty0 + 8 * qb, (uint32_t)((it >> 1) & 1) ^ 1u, ctl, kSiteProdQEmpty))) break;
            if (leader) {
                mbar_arrive_expect_tx(q_full0 + 8 * qb, kQTiles * kTileBytes);
                for (int t = 0; t < kQTiles; ++t)
                    tma_load_3d(q_smem0 + (qb * kQTiles + t) * kTileBytes, &tmQ, q_full0 + 8 * qb, 0,
                                q_row0 + t * kBM, bh);
            }
            last_q = it;
            __syncwarp();
            for (int j = 0; j < nk_item; ++j, ++c) {
                int kv_row, kv_slice;
                kv_coords(p, j, bh, kv_row, kv_slice);
                if (!(ok = warp_wait(k_empty0 + 8 * st, par, ctl, kSiteProdKEmpty))) break;
                if (!p.skip_k_loads) {
                    if (leader) {
                        mbar_arrive_expect_tx(k_full0 + 8 * st, kTileBytes);
                        tma_load_3d(k_smem0 + st * kTileBytes, &tmK, k_full0 + 8 * st, 0, kv_row, kv_slice);
                    }
                    BF_TRACE(3, c, 0);
                    last_k = (int)c;
                }
                if (!(ok = warp_wait(v_empty0 + 8 * st, par, ctl, kSiteProdVEmpty))) break;
                if (leader) {
                    mbar_arrive_expect_tx(v_full0 + 8 * st, kTileBytes);
                    tma_load_3d(v_smem0 + st * kTileBytes, &tmV, v_full0 + 8 * st, 0, kv_row, kv_slice);
                }
                BF_TRACE(3, c, 1);
                last_v = (int)c;
                __syncwarp();
                if (++st == kStages) {
                    st = 0;
                    par ^= 1u;
                }
            }
        }
        if (*ctl.abort_flag) {
            // Let copies still in flight land before the CTA's shared memory is released.
            int never = 0;
            const WaitCtl drain{&never, nullptr, ctl.limit_ns};
            if (last_k >= 0) mbar_wait(k_full0 + 8 * (last_k % kStages), (uint32_t)(last_k / kStages) & 1u, drain, 0);
            if (last_v >= 0) mbar_wait(v_full0 + 8 * (last_v % kStages), (uint32_t)(last_v / kStages) & 1u, drain, 0);
            if (last_q >= 0) mbar_wait(q_full0 + 8 * (last_q & 1), (uint32_t)(last_q >> 1) & 1u, drain, 0);
        }
        __syncwarp();
    } else if (warp == kSWarp || warp == kPVWarp) {
        // ------------------------------------------------------------ MMA issuers
        // Two warps on different schedulers issue the two independent MMA
        // streams: warp kSWarp S_t = Q_t K^T, warp kPVWarp O_t += P_t V. Each
        // whole warp runs its loop (warp-uniform values), waits for all the
        // barriers of a step in one parallel round, and one elected lane issues.
        // Keeping these loops short matters: they share their schedulers with
        // busy softmax warps, and the tensor core's issue queue is shallow.
        constexpr uint32_t kIdescS = idesc_bf16_f32(kBM, kBN, 0);  // Q (K-major) x K (K-major)
        constexpr uint32_t kIdescO = idesc_bf16_f32(kBM, kD, 1);   // P (TMEM)   x V (MN-major)
        const bool leader = elect_one();
        const bool tracing = trace_hit && leader;
        const uint64_t desc_base = smem_desc_sw128(smem_addr(smem), 16, 1024);
        const uint32_t desc_hi = (uint32_t)(desc_base >> 32);
        const uint32_t desc_lo0 = (uint32_t)desc_base;  // low word of a descriptor at smem offset 0
        constexpr uint32_t kTileLo = kTileBytes >> 4;   // low-word step between 16 KiB tiles
        const uint32_t q_lo0 = desc_lo0 + (kOffQ >> 4), k_lo0 = desc_lo0 + (kOffK >> 4), v_lo0 = desc_lo0 + (kOffV >> 4);
        const uint32_t q_full0 = smem_addr(&bars->q_full[0]), q_empty0 = smem_addr(&bars->q_empty[0]);
        const uint32_t k_full0 = smem_addr(&bars->k_full[0]), k_empty0 = smem_addr(&bars->k_empty[0]);
        const uint32_t v_full0 = smem_addr(&bars->v_full[0]), v_empty0 = smem_addr(&bars->v_empty[0]);
        const uint32_t s_full0 = smem_addr(&bars->s_full[0]), s_empty0 = smem_addr(&bars->s_empty[0]);
        const uint32_t p_full0 = smem_addr(&bars->p_full[0]), pv_done0 = smem_addr(&bars->pv_done[0]);
        const bool is_s = warp == kSWarp;

        uint32_t g = 0;          // global KV step
        int st = 0;              // K (S warp) or V (PV warp) stage of step g
        uint32_t par = 0;        // its full-barrier parity
        bool ok = true;
        int it = 0;
        for (int item = blockIdx.x; item < p.items && ok; item += gridDim.x, ++it) {
            const int qb = it & 1;
            int bh_unused, q_row0;
            decode_item(p, item, bh_unused, q_row0);
            const int nk_item = item_kv_tiles(p, q_row0, nk);
            if (is_s) {
                if (!(ok = warp_wait(q_full0 + 8 * qb, (uint32_t)(it >> 1) & 1u, ctl, kSiteMmaQ))) break;
                tc_fence_after();
            }
            for (int j = 0; j < nk_item; ++j, ++g) {
                if (is_s) {
                    // K(g) loaded; then each S_t is issued as soon as its softmax has read S_t(g-1),
                    // so the two tiles may run half a step apart (ping-pong).
                    if (!(ok = warp_wait(k_full0 + 8 * st, par, ctl, kSiteMmaK))) break;
                    tc_fence_after();
                    BF_TRACE(2, g, 0);
                    const uint32_t k_lo = k_lo0 + (uint32_t)st * kTileLo;
#pragma unroll
                    for (int t = 0; t < kQTiles; ++t) {
                        if (g > 0) {
                            if (!(ok = warp_wait(s_empty0 + 8 * t, (g - 1) & 1u, ctl, kSiteMmaK + 1 + t))) break;
                            tc_fence_after();
                        }
                        BF_TRACE(2, g, 4 + t);  // S_t(g) issue starts
                        if (leader) {
                            const uint32_t q_lo = q_lo0 + (uint32_t)(qb * kQTiles + t) * kTileLo;
#pragma unroll
                            for (int kk = 0; kk < kD / 16; ++kk)  // 16 head-dim elements = 32 B inside the swizzle atom
                                umma_ss_lo(tmem + kColS + t * kBN, q_lo + kk * 2, k_lo + kk * 2, desc_hi, kIdescS, kk > 0);
                            umma_commit(s_full0 + 8 * t);
                        }
                        __syncwarp();
                    }
                    if (!ok) break;
                    if (leader) {
                        umma_commit(k_empty0 + 8 * st);
                        if (j == nk_item - 1) umma_commit(q_empty0 + 8 * qb);  // last S of this item: Q buffer free
                    }
                    __syncwarp();
                    BF_TRACE(2, g, 1);
                } else {
                    // V(g) loaded; then each PV_t as soon as P_t(g) is written.
                    if (!(ok = warp_wait(v_full0 + 8 * st, par, ctl, kSiteMmaV))) break;
                    BF_TRACE(2, g, 2);
                    const uint32_t v_lo = v_lo0 + (uint32_t)st * kTileLo;
#pragma unroll
                    for (int t = 0; t < kQTiles; ++t) {
                        if (!(ok = warp_wait(p_full0 + 8 * t, g & 1u, ctl, kSiteMmaV + 1 + t))) break;
                        tc_fence_after();
                        BF_TRACE(2, g, 6 + t);  // PV_t(g) issue starts
                        if (leader) {
                            const uint32_t p_col = tmem + kColP + t * kD;
#pragma unroll
                            for (int kk = 0; kk < kBN / 16; ++kk)  // 16 KV rows: 8 TMEM columns of P, 16 x 128 B of V
                                umma_ts_lo(tmem + kColO + t * kD, p_col + kk * 8, v_lo + kk * 128, desc_hi, kIdescO,
                                           (j > 0 || kk > 0) ? 1u : 0u);
                            umma_commit(pv_done0 + 8 * t);
                        }
                        __syncwarp();
                    }
                    if (!ok) break;
                    if (leader) umma_commit(v_empty0 + 8 * st);
                    __syncwarp();
                    BF_TRACE(2, g, 3);
                }
                if (++st == kStages) {
                    st = 0;
                    par ^= 1u;
                }
            }
        }
        // Drain: every MMA this warp issued has finished before TMEM is released.
        const uint32_t drain_bar = smem_addr(is_s ? &bars->drain : &bars->drain_pv);
        if (leader) umma_commit(drain_bar);
        __syncwarp();
        int never = 0;
        const WaitCtl drain{&never, nullptr, ctl.limit_ns};
        mbar_wait(drain_bar, 0u, drain, 0);
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kSWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    if constexpr (kTrace) {
        if (threadIdx.x == 0) p.trace[4 * 512 + blockIdx.x * 4 + 3] = (long long)global_timer_ns();
    }
}

#include "fa_fwd_sm100_d128.cuh"
#include "fa_bwd_sm100.cuh"

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
// For d = 128 the same 64-column box is loaded twice per tile (columns 0 and 64).
int make_map(CUtensorMap* m, const void* base, long long bh, int rows, int d = bfk::kD) {
    PFN_encodeTiled enc = get_encode_fn();
    if (!enc) return bf_set_error(BF_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    // The encode is a driver call and needs a current context. A thread that has only
    // used the runtime implicitly (torch's autograd worker, for one) may not have one
    // yet; cudaSetDevice makes the device's primary context current.
    int cur = 0;
    if (cudaGetDevice(&cur) != cudaSuccess || cudaSetDevice(cur) != cudaSuccess)
        return bf_set_error(BF_ERR_CUDA, "no CUDA device context");
    cuuint64_t dims[3] = {(cuuint64_t)d, (cuuint64_t)rows, (cuuint64_t)bh};
    cuuint64_t strides[2] = {(cuuint64_t)d * 2, (cuuint64_t)rows * d * 2};
    cuuint32_t box[3] = {(cuuint32_t)bfk::kD, (cuuint32_t)bfk::kBM, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char msg[200];
        snprintf(msg, sizeof(msg), "cuTensorMapEncodeTiled rejected the tensor (error %d, base %p, rows %d, slices %lld, d %d)",
                 (int)r, base, rows, bh, d);
        return bf_set_error(BF_ERR_CUDA, msg);
    }
    return BF_OK;
}

// Tensor maps depend only on (base, slices, rows, d); the launchers ask for four per
// call, and the encode is a driver call, so the last few are kept per host thread and
// per device.
struct MapCacheEntry {
    const void* base;
    long long bh;
    int rows, d, dev;
    CUtensorMap map;
};
constexpr int kMapCacheSize = 16;
thread_local MapCacheEntry g_map_cache[kMapCacheSize];
thread_local int g_map_cache_used = 0, g_map_cache_next = 0;

int cached_map(CUtensorMap* m, const void* base, long long bh, int rows, int d = bfk::kD) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return bf_set_error(BF_ERR_CUDA, "cudaGetDevice failed");
    for (int i = 0; i < g_map_cache_used; ++i) {
        const MapCacheEntry& e = g_map_cache[i];
        if (e.base == base && e.bh == bh && e.rows == rows && e.d == d && e.dev == dev) {
            *m = e.map;
            return BF_OK;
        }
    }
    const int rc = make_map(m, base, bh, rows, d);
    if (rc != BF_OK) return rc;
    MapCacheEntry& e = g_map_cache[g_map_cache_next];
    e.base = base;
    e.bh = bh;
    e.rows = rows;
    e.d = d;
    e.dev = dev;
    e.map = *m;
    g_map_cache_next = (g_map_cache_next + 1) % kMapCacheSize;
    if (g_map_cache_used < kMapCacheSize) ++g_map_cache_used;
    return BF_OK;
}

// Launch with programmatic stream serialisation: the kernel's set-up overlaps the tail
// of the previous kernel on the stream (the kernels wait with griddepcontrol.wait
// before touching global memory).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), unsigned grid, unsigned block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    // BLACKFLASH_NO_PDL=1 launches with plain stream order (read once per process).
    static const bool no_pdl = [] {
        const char* v = getenv("BLACKFLASH_NO_PDL");
        return v && v[0] && v[0] != '0';
    }();
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = no_pdl ? 0 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <bool kF32Out>
int configure_once() {
    static std::atomic<bool> done[64];  // per device; zero-initialised (static storage)
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

int sm_count(int* out) {
    static std::atomic<int> cached[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return bf_set_error(BF_ERR_CUDA, "cudaGetDevice failed");
    if (!cached[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            return bf_set_error(BF_ERR_CUDA, "cannot query the SM count");
        cached[dev] = n;
    }
    *out = cached[dev];
    return BF_OK;
}

int bf_fwd_launch(const BfFwdArgs* a) {
    int rc0;
    if (a->d != bfk::kD && a->d != bfk::d128::kD) return bf_set_error(BF_ERR_ARG, "BlackFlash supports d=64 and d=128");
    if (a->bh <= 0 || a->n_q <= 0 || a->n_kv <= 0) return bf_set_error(BF_ERR_ARG, "empty problem: B*H and N must be >= 1");
    if (!a->q || !a->k || !a->v || (!a->o && !a->o_f32)) return bf_set_error(BF_ERR_ARG, "null tensor pointer");
    auto misaligned = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) != 0; };
    if (misaligned(a->q) || misaligned(a->k) || misaligned(a->v) || (a->o && misaligned(a->o)) ||
        (a->o_f32 && misaligned(a->o_f32)))
        return bf_set_error(BF_ERR_ARG, "Q/K/V/O must be 16-byte aligned");
    const long long q_blocks = (a->n_q + bfk::kQTiles * bfk::kBM - 1) / (bfk::kQTiles * bfk::kBM);
    const long long items = q_blocks * a->bh;
    if (items > 0x7fffffffLL || a->bh > 0x7fffffffLL) return bf_set_error(BF_ERR_ARG, "problem too large for one launch");
    int sms = 0;
    if ((rc0 = sm_count(&sms)) != BF_OK) return rc0;
    const long long grid = items < sms ? items : sms;  // persistent: at most one CTA per SM

    CUtensorMap mq, mk, mv, mo;
    int rc;
    if (a->d == bfk::d128::kD) {
        if (!a->o || a->o_f32 || a->kv_blocks || a->trace || a->dbg_s || a->skip_k_loads)
            return bf_set_error(BF_ERR_ARG, "d=128 supports the bf16 forward (causal, lse and row max optional) only");
        if ((rc = cached_map(&mq, a->q, a->bh, a->n_q, 128)) != BF_OK) return rc;
        if ((rc = cached_map(&mk, a->k, a->bh, a->n_kv, 128)) != BF_OK) return rc;
        if ((rc = cached_map(&mv, a->v, a->bh, a->n_kv, 128)) != BF_OK) return rc;
        bfk::KParams kp;
        memset(&kp, 0, sizeof(kp));
        kp.n_q = a->n_q;
        kp.n_kv = a->n_kv;
        kp.q_blocks = (int)q_blocks;
        kp.items = (int)items;
        kp.scale = a->scale;
        kp.scale_log2 = a->scale * 1.4426950408889634f;
        kp.lse = a->lse;
        kp.row_max = a->row_max;
        kp.timeout_ns = a->timeout_ns ? a->timeout_ns : 4000000000ull;
        kp.causal = a->causal;
        kp.kv_skip = -1;
        kp.bh_count = (int)a->bh;
        static std::atomic<bool> done[64];  // per device; zero-initialised (static storage)
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return bf_set_error(BF_ERR_CUDA, "cudaGetDevice failed");
        if (!done[dev]) {
            cudaError_t e = cudaFuncSetAttribute(bfk::d128::fa_fwd_d128_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 bfk::d128::kSmemBytes);
            if (e != cudaSuccess) return bf_set_error(BF_ERR_CUDA, cudaGetErrorString(e));
            done[dev] = true;
        }
        const cudaError_t e =
            launch_pdl(bfk::d128::fa_fwd_d128_kernel, (unsigned)grid, bfk::kThreads, bfk::d128::kSmemBytes,
                       reinterpret_cast<cudaStream_t>(a->stream), mq, mk, mv, reinterpret_cast<__nv_bfloat16*>(a->o), kp);
        if (e != cudaSuccess) return bf_set_error(BF_ERR_CUDA, cudaGetErrorString(e));
        return BF_OK;
    }
    if ((rc = cached_map(&mq, a->q, a->bh, a->n_q)) != BF_OK) return rc;
    int kv_blk_tiles = 0;
    if (a->kv_blocks) {
        if (a->kv_blocks < 1 || a->kv_block_rows <= 0 || a->kv_block_rows % bfk::kBN ||
            a->kv_skip < -1 || a->kv_skip >= a->kv_blocks || a->causal)
            return bf_set_error(BF_ERR_ARG, "blocked KV needs block rows % 128 == 0, -1 <= skip < blocks, non-causal");
        if (a->n_kv != (a->kv_blocks - (a->kv_skip >= 0)) * (long long)a->kv_block_rows)
            return bf_set_error(BF_ERR_ARG, "blocked KV: n_kv must equal the rows of the blocks used");
        if ((long long)a->kv_blocks * a->bh > 0x7fffffffLL) return bf_set_error(BF_ERR_ARG, "problem too large for one launch");
        kv_blk_tiles = a->kv_block_rows / bfk::kBN;
        if ((rc = cached_map(&mk, a->k, (long long)a->kv_blocks * a->bh, a->kv_block_rows)) != BF_OK) return rc;
        if ((rc = cached_map(&mv, a->v, (long long)a->kv_blocks * a->bh, a->kv_block_rows)) != BF_OK) return rc;
    } else {
        if ((rc = cached_map(&mk, a->k, a->bh, a->n_kv)) != BF_OK) return rc;
        if ((rc = cached_map(&mv, a->v, a->bh, a->n_kv)) != BF_OK) return rc;
    }
    if (a->o) {
        if ((rc = cached_map(&mo, a->o, a->bh, a->n_q)) != BF_OK) return rc;
    } else {
        mo = mq;  // not read in fp32-output mode
    }

    bfk::KParams kp;
    kp.n_q = a->n_q;
    kp.n_kv = a->n_kv;
    kp.q_blocks = (int)q_blocks;
    kp.items = (int)items;
    kp.scale = a->scale;
    kp.scale_log2 = a->scale * 1.4426950408889634f;
    kp.lse = a->lse;
    kp.row_max = a->row_max;
    kp.o_f32 = a->o_f32;
    kp.timeout_ns = a->timeout_ns ? a->timeout_ns : 4000000000ull;
    kp.dbg_s = a->dbg_s;
    kp.skip_k_loads = a->skip_k_loads;
    kp.trace = a->trace;
    kp.causal = a->causal;
    kp.trace_cta = a->trace_cta;
    kp.kv_blk_tiles = kv_blk_tiles;
    kp.kv_skip = a->kv_blocks ? a->kv_skip : -1;
    kp.bh_count = (int)a->bh;

    cudaStream_t stream = reinterpret_cast<cudaStream_t>(a->stream);
    if (a->trace) {
        if (a->o_f32) return bf_set_error(BF_ERR_ARG, "trace runs use the bf16 output");
        static std::atomic<bool> traced_cfg[64];
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev >= 0 && dev < 64 && !traced_cfg[dev]) {
            cudaFuncSetAttribute(bfk::fa_fwd_sm100_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 bfk::kSmemBytes);
            traced_cfg[dev] = true;
        }
        bfk::fa_fwd_sm100_kernel<false, true><<<(unsigned)grid, bfk::kThreads, bfk::kSmemBytes, stream>>>(mq, mk, mv, mo, kp);
    } else if (a->o_f32) {
        if ((rc = configure_once<true>()) != BF_OK) return rc;
        const cudaError_t e = launch_pdl(bfk::fa_fwd_sm100_kernel<true>, (unsigned)grid, bfk::kThreads, bfk::kSmemBytes,
                                         stream, mq, mk, mv, mo, kp);
        if (e != cudaSuccess) return bf_set_error(BF_ERR_CUDA, cudaGetErrorString(e));
    } else {
        if ((rc = configure_once<false>()) != BF_OK) return rc;
        const cudaError_t e = launch_pdl(bfk::fa_fwd_sm100_kernel<false>, (unsigned)grid, bfk::kThreads,
                                         bfk::kSmemBytes, stream, mq, mk, mv, mo, kp);
        if (e != cudaSuccess) return bf_set_error(BF_ERR_CUDA, cudaGetErrorString(e));
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return bf_set_error(BF_ERR_CUDA, cudaGetErrorString(e));
    return BF_OK;
}

long long bf_bwd_workspace_bytes(long long bh, int n) {
    const long long n_pad = ((long long)n + 127) / 128 * 128;
    return 4LL * (bh * n * 64 + 2 * bh * n_pad);
}

int bf_bwd_launch(const BfBwdArgs* a) {
    if (a->d != bfk::kD) return bf_set_error(BF_ERR_ARG, "the backward supports d=64");
    if (a->bh <= 0 || a->n <= 0) return bf_set_error(BF_ERR_ARG, "empty problem: B*H and N must be >= 1");
    const void* ptrs[] = {a->q, a->k, a->v, a->o, a->dout, a->lse, a->dq, a->dk, a->dv, a->workspace};
    for (const void* ptr : ptrs) {
        if (!ptr) return bf_set_error(BF_ERR_ARG, "null pointer");
        if (reinterpret_cast<uintptr_t>(ptr) & 15u) return bf_set_error(BF_ERR_ARG, "every pointer must be 16-byte aligned");
    }
    const long long q_tiles = ((long long)a->n + 127) / 128;
    const long long blocks = q_tiles * a->bh;
    if (blocks > 0x7fffffffLL) return bf_set_error(BF_ERR_ARG, "problem too large for one launch");
    const int n_pad = (int)(q_tiles * 128);
    float* dq_acc = reinterpret_cast<float*>(a->workspace);
    float* dvec = dq_acc + (size_t)a->bh * a->n * 64;
    float* lse2 = dvec + (size_t)a->bh * n_pad;
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(a->stream);

    CUtensorMap mq, mk, mv, mdo;
    int rc;
    if ((rc = make_map(&mq, a->q, a->bh, a->n)) != BF_OK) return rc;
    if ((rc = make_map(&mk, a->k, a->bh, a->n)) != BF_OK) return rc;
    if ((rc = make_map(&mv, a->v, a->bh, a->n)) != BF_OK) return rc;
    if ((rc = make_map(&mdo, a->dout, a->bh, a->n)) != BF_OK) return rc;
    // The fp32 dQ accumulator [BH][n][64] as a 3-D map for the kernel's TMA reduce-adds:
    // 32-column (128-byte) x 128-row boxes with 128-byte swizzle; rows past n are clipped.
    CUtensorMap mdq;
    {
        PFN_encodeTiled enc = get_encode_fn();
        if (!enc) return bf_set_error(BF_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
        cuuint64_t dims[3] = {64, (cuuint64_t)a->n, (cuuint64_t)a->bh};
        cuuint64_t strides[2] = {64 * 4, (cuuint64_t)a->n * 64 * 4};
        cuuint32_t box[3] = {32, 128, 1};
        cuuint32_t estr[3] = {1, 1, 1};
        const CUresult r = enc(&mdq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, dq_acc, dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return bf_set_error(BF_ERR_CUDA, "cuTensorMapEncodeTiled rejected the dQ accumulator");
    }
    static std::atomic<bool> done[64];  // per device; zero-initialised (static storage)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return bf_set_error(BF_ERR_CUDA, "cudaGetDevice failed");
    if (!done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(bfk::bwd::fa_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             bfk::bwd::kSmemBytesB);
        if (e != cudaSuccess) return bf_set_error(BF_ERR_CUDA, cudaGetErrorString(e));
        done[dev] = true;
    }
    int sms = 0;
    if ((rc = sm_count(&sms)) != BF_OK) return rc;

    cudaError_t e = cudaMemsetAsync(dq_acc, 0, sizeof(float) * (size_t)a->bh * a->n * 64, stream);
    if (e != cudaSuccess) return bf_set_error(BF_ERR_CUDA, cudaGetErrorString(e));
    auto launch_err = [](const char* what) -> int {
        const cudaError_t le = cudaGetLastError();
        if (le == cudaSuccess) return BF_OK;
        char msg[256];
        snprintf(msg, sizeof(msg), "%s: %s", what, cudaGetErrorString(le));
        return bf_set_error(BF_ERR_CUDA, msg);
    };
    if ((rc = launch_err("before the backward")) != BF_OK) return rc;
    bfk::bwd::bwd_prep_kernel<<<sms * 8, 256, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(a->o), reinterpret_cast<const __nv_bfloat16*>(a->dout), a->lse, dvec,
        lse2, a->bh, a->n, n_pad);
    bfk::bwd::BParams bp;
    bp.n = a->n;
    bp.n_pad = n_pad;
    bp.q_tiles = (int)q_tiles;
    bp.scale = a->scale;
    bp.scale_log2 = a->scale * 1.4426950408889634f;
    bp.lse2 = lse2;
    bp.dvec = dvec;
    bp.dq_acc = dq_acc;
    bp.dk = reinterpret_cast<__nv_bfloat16*>(a->dk);
    bp.dv = reinterpret_cast<__nv_bfloat16*>(a->dv);
    bp.timeout_ns = a->timeout_ns ? a->timeout_ns : 4000000000ull;
    if ((rc = launch_err("backward prep kernel")) != BF_OK) return rc;
    bfk::bwd::fa_bwd_kernel<<<(unsigned)blocks, bfk::bwd::kThreadsB, bfk::bwd::kSmemBytesB, stream>>>(mq, mk, mv, mdo, mdq, bp);
    {
        const cudaError_t le = cudaGetLastError();
        if (le != cudaSuccess) {
            cudaFuncAttributes fa;
            cudaFuncGetAttributes(&fa, bfk::bwd::fa_bwd_kernel);
            char msg[256];
            snprintf(msg, sizeof(msg), "backward kernel: %s (regs %d, max threads %d, local %zu B, smem %d B)",
                     cudaGetErrorString(le), fa.numRegs, fa.maxThreadsPerBlock, fa.localSizeBytes, bfk::bwd::kSmemBytesB);
            return bf_set_error(BF_ERR_CUDA, msg);
        }
    }
    bfk::bwd::bwd_dq_kernel<<<sms * 8, 256, 0, stream>>>(dq_acc, reinterpret_cast<__nv_bfloat16*>(a->dq), a->scale,
                                                          (size_t)a->bh * a->n * 16);
    e = cudaGetLastError();
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
