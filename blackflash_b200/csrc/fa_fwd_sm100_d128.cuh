// Head dimension 128 variant of the sm_100a forward (included by fa_fwd_sm100.cu,
// inside namespace bfk, after KParams / decode_item / item_kv_tiles / g_wait_status).
//
// Same work decomposition as the d = 64 kernel (persistent CTAs, items of two
// 128-row query tiles, 16 softmax warps with two threads per row, a TMA producer
// and two MMA issuer warps), with the resources rearranged for d = 128:
//
//   TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512).
//     O now needs 128 columns per tile, so there is no separate P buffer: the
//     softmax writes bf16 P_t over the first 64 columns of S_t (it has already
//     loaded S_t into registers). S_t(g+1) is therefore issued only after
//     PV_t(g) has read P_t(g) (pv_done_t), which also guarantees that O_t is
//     stable whenever the softmax rescales it - the softmax itself never waits
//     for a PV. The two tiles alternate naturally: while one waits for its
//     PV + S, the other runs its exponentials.
//   Shared memory (192 KiB + barriers): Q one buffer per tile (2 x 32 KiB),
//     released after the tile's last S of the item, so the next item's Q_t
//     loads while the other tile finishes; K and V 2 stages x 32 KiB each.
//     Each 128-column tile is two 64-column chunks of 128-byte-swizzled rows
//     (one TMA box each); S = Q K^T runs K = 128 as 8 K16 steps across the two
//     chunks, and PV is two N = 64 MMAs per K16 step, one per V chunk.
//   Epilogue: O_t is scaled by 1/l and written to global memory straight from
//     registers (no staging buffer: shared memory is full).
namespace d128 {

constexpr int kD = 128;
constexpr int kChunk = 64;                       // columns per 128-byte swizzle span
constexpr int kChunkBytes = 128 * kChunk * 2;    // 16 KiB: 128 rows x 64 bf16
constexpr int kTileBytes = 2 * kChunkBytes;      // 32 KiB: one 128 x 128 bf16 tile
constexpr int kStages = 2;
constexpr int kOffQ = 0;                                 // [2 tiles][2 chunks]
constexpr int kOffK = kOffQ + kQTiles * kTileBytes;      // [kStages][2 chunks]
constexpr int kOffV = kOffK + kStages * kTileBytes;      // [kStages][2 chunks]
constexpr int kOffBar = kOffV + kStages * kTileBytes;
constexpr int kColO = 2 * kBN;                           // O_t at 256 + 128 t
constexpr int kHalfN = 64;                               // S is issued as two N = 64 halves
// At d = 128 the tensor core carries twice the work per exponential, so MUFU has
// headroom and the FMA-pipe exp2 only costs issue slots: measured best at 0 of 8.
#ifndef BF_EMU_PAIRS_D128
#define BF_EMU_PAIRS_D128 0
#endif
constexpr int kEmuPairs128 = BF_EMU_PAIRS_D128;          // FMA-pipe exp2 pairs of every kEmuPeriod

struct Bars {
    uint64_t q_full[kQTiles];
    uint64_t q_empty[kQTiles];
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
constexpr int kSmemBytes = kOffBar + (int)sizeof(Bars) + 1024;
static_assert(kSmemBytes <= 227 * 1024, "shared memory");

enum : unsigned {
    kSiteProdQ = 0x500,
    kSiteProdK = 0x501,
    kSiteProdV = 0x502,
    kSiteMmaQ = 0x510,  // + t
    kSiteMmaK = 0x520,  // +0 K full, +1 + t PV_t(g-1) done, +3 + t S_t(g-1) loaded
    kSiteMmaV = 0x530,  // +0 V full, +1 + t P_t full
    kSiteSoftS = 0x540,
    kSiteSoftO = 0x541,
};

__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_d128_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ out, const KParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nk = (p.n_kv + kBN - 1) / kBN;

    if (threadIdx.x == 0) {
        for (int t = 0; t < kQTiles; ++t) {
            mbar_init(smem_addr(&bars->q_full[t]), 1);
            mbar_init(smem_addr(&bars->q_empty[t]), 1);
            mbar_init(smem_addr(&bars->s_full[t]), 1);
            mbar_init(smem_addr(&bars->s_empty[t]), 2 * kBM);
            mbar_init(smem_addr(&bars->p_full[t]), 2 * kBM);
            mbar_init(smem_addr(&bars->pv_done[t]), 1);
        }
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_addr(&bars->k_full[s]), 1);
            mbar_init(smem_addr(&bars->k_empty[s]), 1);
            mbar_init(smem_addr(&bars->v_full[s]), 1);
            mbar_init(smem_addr(&bars->v_empty[s]), 1);
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

#if BF_REGSPLIT
    if (warp < kSoftWarps)
        regs_inc<104>();
    else
        regs_dec<64>();
#endif
    if (warp < kSoftWarps) {
        // ------------------------------------------------------------ softmax
        // Row layout as in the d = 64 kernel: warp w of tile t covers 16 TMEM
        // lanes; lanes i and i + 16 share a row, one per 64-column half of S.
        const int t = warp >> 3;
        const int quarter = warp & 3;
        const int sub = (warp >> 2) & 1;
        const int h = lane >> 4;
        const int row = quarter * 32 + sub * 16 + (lane & 15);
        const uint32_t lane_off = (uint32_t)(quarter * 32 + sub * 16) << 16;
        const uint32_t tS = tmem + lane_off + (uint32_t)(t * kBN);
        const uint32_t tP = tS;  // bf16 P over the first 64 columns of S_t
        const uint32_t tO = tmem + lane_off + (uint32_t)(kColO + t * kD);
        const float sl2 = p.scale_log2;
        const uint64_t sl2_2 = f2_pack(sl2, sl2);
        const uint32_t bar_s = smem_addr(&bars->s_full[t]);
        const uint32_t bar_se = smem_addr(&bars->s_empty[t]);
        const uint32_t bar_p = smem_addr(&bars->p_full[t]);
        const uint32_t bar_pv = smem_addr(&bars->pv_done[t]);
        uint32_t g = 0;
        bool ok = true;

        for (int item = blockIdx.x; item < p.items && ok; item += gridDim.x) {
            int bh, q_row0;
            decode_item(p, item, bh, q_row0);
            const int nk_item = item_kv_tiles(p, q_row0, nk);
            float m_use = -INFINITY;
            float m_raw = -INFINITY;
            float l_half = 0.f;

            for (int j = 0; j < nk_item; ++j, ++g) {
                if (!(ok = warp_wait(bar_s, g & 1u, ctl, kSiteSoftS))) break;
                tc_fence_after();
                uint32_t s[2][32];
                tmem_ld16x32bx2_x32<64>(tS + 0, s[0]);
                tmem_ld16x32bx2_x32<64>(tS + 32, s[1]);
                tmem_wait_ld();
                tc_fence_before();
                mbar_arrive(bar_se);  // S_t is in registers: its upper 64 columns may be rewritten

                const int q_abs = q_row0 + t * kBM + row;
                const int kv_lim = p.causal ? min(p.n_kv, q_abs + 1) : p.n_kv;
                const int valid = kv_lim - j * kBN - h * 64;
                if (valid < 64) {
#pragma unroll
                    for (int c = 0; c < 64; ++c)
                        if (c >= valid) s[c >> 5][c & 31] = __float_as_uint(-INFINITY);
                }

                float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
                for (int c = 0; c < 32; c += 2) {
                    mx0 = fmax3(mx0, __uint_as_float(s[0][c]), __uint_as_float(s[0][c + 1]));
                    mx1 = fmax3(mx1, __uint_as_float(s[1][c]), __uint_as_float(s[1][c + 1]));
                }
                float mx = fmaxf(mx0, mx1);
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                m_raw = fmaxf(m_raw, mx);
                const float m_new = mx * sl2;
                float alpha = 1.f;
                const bool need = m_new > m_use + 8.0f;  // lazy rescale, as in the d = 64 kernel
                if (need) {
                    alpha = fast_exp2(m_use - m_new);
                    m_use = m_new;
                }

                uint32_t pk[2][16];
                const uint64_t negm_2 = f2_pack(-m_use, -m_use);
                uint64_t sum_a = f2_pack(0.f, 0.f), sum_b = f2_pack(0.f, 0.f);
#pragma unroll
                for (int q = 0; q < 2; ++q) {
#pragma unroll
                    for (int c = 0; c < 16; ++c) {
                        const uint64_t x2 =
                            f2_fma(f2_pack(__uint_as_float(s[q][2 * c]), __uint_as_float(s[q][2 * c + 1])), sl2_2, negm_2);
                        uint64_t p2;
                        if (((q * 16 + c) & (kEmuPeriod - 1)) < kEmuPairs128) {
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
                {
                    float a0, a1, b0, b1;
                    f2_unpack(sum_a, a0, a1);
                    f2_unpack(sum_b, b0, b1);
                    l_half = l_half * alpha + ((a0 + a1) + (b0 + b1));
                }

                // PV_t(g-1) finished before S_t(g) was issued, so O_t is stable here.
                if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll 1
                    for (int half = 0; half < 2; ++half) {
                        uint32_t o[32];  // O columns 64h + 32 half + [0, 32)
                        tmem_ld16x32bx2_x32<64>(tO + 32 * half, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
                        tmem_st16x32bx2_x32<64>(tO + 32 * half, o);
                    }
                }
                // bf16 P: this thread's 64 keys are P columns 32h + [0, 32).
                tmem_st16x32bx2_x16<32>(tP, pk[0]);
                tmem_st16x32bx2_x16<32>(tP + 16, pk[1]);
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(bar_p);
            }
            if (!ok) break;

            // ---------------------------------------------------- epilogue of this item
            if (!(ok = warp_wait(bar_pv, (g - 1) & 1u, ctl, kSiteSoftO))) break;
            tc_fence_after();
            const float l_sum = l_half + __shfl_xor_sync(0xffffffffu, l_half, 16);
            const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
            const int q_row = q_row0 + t * kBM + row;
            const bool row_ok = q_row < p.n_q;
#pragma unroll 1
            for (int half = 0; half < 2; ++half) {
                uint32_t o[32];
                tmem_ld16x32bx2_x32<64>(tO + 32 * half, o);
                tmem_wait_ld();
                if (row_ok) {
                    uint4* dst = reinterpret_cast<uint4*>(out + ((size_t)bh * p.n_q + q_row) * kD + h * 64 + half * 32);
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint32_t* src = &o[c * 8];
                        uint4 v;
                        v.x = pack_bf16x2(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv);
                        v.y = pack_bf16x2(__uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv);
                        v.z = pack_bf16x2(__uint_as_float(src[4]) * inv, __uint_as_float(src[5]) * inv);
                        v.w = pack_bf16x2(__uint_as_float(src[6]) * inv, __uint_as_float(src[7]) * inv);
                        dst[c] = v;
                    }
                }
            }
            // The next item's first PV overwrites O_t: every load above has completed
            // (wait::ld) before this thread arrives on p_full again.
            if (row_ok && h == 0) {
                const size_t idx = (size_t)bh * p.n_q + q_row;
                if (p.lse) p.lse[idx] = (m_use + __log2f(l_sum)) * 0.69314718055994531f;
                if (p.row_max) p.row_max[idx] = m_raw * p.scale;
            }
        }
    } else if (warp == kProducerWarp) {
        // ------------------------------------------------------------ TMA producer
        const bool leader = elect_one();
        const uint32_t q_smem0 = smem_addr(smem + kOffQ);
        const uint32_t k_smem0 = smem_addr(smem + kOffK), v_smem0 = smem_addr(smem + kOffV);
        int last_k = -1, last_v = -1, last_q = -1;
        uint32_t c = 0;
        int st = 0;
        uint32_t par = 1u;
        bool ok = true;
        int it = 0;
        for (int item = blockIdx.x; item < p.items && ok; item += gridDim.x, ++it) {
            int bh, q_row0;
            decode_item(p, item, bh, q_row0);
            const int nk_item = item_kv_tiles(p, q_row0, nk);
            // Q_0 first; Q_1 after the item's first K/V tile, so K(0) does not wait for the
            // previous item's last S_1 (which frees Q_1's buffer).
            auto load_q = [&](int t) -> bool {
                const uint32_t qf = smem_addr(&bars->q_full[t]);
                if (!warp_wait(smem_addr(&bars->q_empty[t]), (uint32_t)(it & 1) ^ 1u, ctl, kSiteProdQ)) return false;
                if (leader) {
                    mbar_arrive_expect_tx(qf, kTileBytes);
                    for (int ch = 0; ch < 2; ++ch)
                        tma_load_3d(q_smem0 + t * kTileBytes + ch * kChunkBytes, &tmQ, qf, ch * kChunk,
                                    q_row0 + t * kBM, bh);
                }
                __syncwarp();
                return true;
            };
            if (!(ok = load_q(0))) break;
            last_q = it;
            for (int j = 0; j < nk_item; ++j, ++c) {
                const uint32_t kf = smem_addr(&bars->k_full[st]), vf = smem_addr(&bars->v_full[st]);
                if (!(ok = warp_wait(smem_addr(&bars->k_empty[st]), par, ctl, kSiteProdK))) break;
                if (leader) {
                    mbar_arrive_expect_tx(kf, kTileBytes);
                    for (int ch = 0; ch < 2; ++ch)
                        tma_load_3d(k_smem0 + st * kTileBytes + ch * kChunkBytes, &tmK, kf, ch * kChunk, j * kBN, bh);
                }
                last_k = (int)c;
                if (!(ok = warp_wait(smem_addr(&bars->v_empty[st]), par, ctl, kSiteProdV))) break;
                if (leader) {
                    mbar_arrive_expect_tx(vf, kTileBytes);
                    for (int ch = 0; ch < 2; ++ch)
                        tma_load_3d(v_smem0 + st * kTileBytes + ch * kChunkBytes, &tmV, vf, ch * kChunk, j * kBN, bh);
                }
                last_v = (int)c;
                __syncwarp();
                if (j == 0 && !(ok = load_q(1))) break;
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
            if (last_k >= 0)
                mbar_wait(smem_addr(&bars->k_full[last_k % kStages]), (uint32_t)(last_k / kStages) & 1u, drain, 0);
            if (last_v >= 0)
                mbar_wait(smem_addr(&bars->v_full[last_v % kStages]), (uint32_t)(last_v / kStages) & 1u, drain, 0);
            if (last_q >= 0)
                for (int t = 0; t < kQTiles; ++t) mbar_wait(smem_addr(&bars->q_full[t]), (uint32_t)last_q & 1u, drain, 0);
        }
        __syncwarp();
    } else if (warp == kSWarp || warp == kPVWarp) {
        // ------------------------------------------------------------ MMA issuers
        constexpr uint32_t kIdescSh = idesc_bf16_f32(kBM, kHalfN, 0);  // Q (K-major) x 64 K rows (K-major)
        constexpr uint32_t kHalfRowsLo = (64 * 128) >> 4;             // K rows 64.. inside a chunk
        constexpr uint32_t kIdescO = idesc_bf16_f32(kBM, kChunk, 1);  // P (TMEM)   x V chunk (MN-major)
        const bool leader = elect_one();
        const uint64_t desc_base = smem_desc_sw128(smem_addr(smem), 16, 1024);
        const uint32_t desc_hi = (uint32_t)(desc_base >> 32);
        const uint32_t desc_lo0 = (uint32_t)desc_base;
        constexpr uint32_t kChunkLo = kChunkBytes >> 4;
        constexpr uint32_t kTileLo = kTileBytes >> 4;
        const uint32_t q_lo0 = desc_lo0 + (kOffQ >> 4), k_lo0 = desc_lo0 + (kOffK >> 4), v_lo0 = desc_lo0 + (kOffV >> 4);
        const bool is_s = warp == kSWarp;
        uint32_t g = 0;
        int st = 0;
        uint32_t par = 0;
        bool ok = true;
        int it = 0;
        for (int item = blockIdx.x; item < p.items && ok; item += gridDim.x, ++it) {
            int bh_unused, q_row0;
            decode_item(p, item, bh_unused, q_row0);
            const int nk_item = item_kv_tiles(p, q_row0, nk);
            for (int j = 0; j < nk_item; ++j, ++g) {
                if (is_s) {
                    if (!(ok = warp_wait(smem_addr(&bars->k_full[st]), par, ctl, kSiteMmaK))) break;
                    tc_fence_after();
                    const uint32_t k_lo = k_lo0 + (uint32_t)st * kTileLo;
#pragma unroll
                    for (int t = 0; t < kQTiles; ++t) {
                        if (j == 0) {  // this item's Q_t
                            if (!(ok = warp_wait(smem_addr(&bars->q_full[t]), (uint32_t)it & 1u, ctl, kSiteMmaQ + t)))
                                break;
                            tc_fence_after();
                        }
                        const uint32_t q_lo = q_lo0 + (uint32_t)t * kTileLo;
                        // Upper half (keys 64..127 -> S_t columns 64..127): free once the
                        // softmax has loaded S_t(g-1).
                        if (g > 0) {
                            if (!(ok = warp_wait(smem_addr(&bars->s_empty[t]), (g - 1) & 1u, ctl, kSiteMmaK + 3 + t)))
                                break;
                            tc_fence_after();
                        }
                        if (leader) {
#pragma unroll
                            for (int kk = 0; kk < kD / 16; ++kk) {
                                const uint32_t off = (uint32_t)(kk >> 2) * kChunkLo + (uint32_t)(kk & 3) * 2;
                                umma_ss_lo(tmem + t * kBN + kHalfN, q_lo + off, k_lo + off + kHalfRowsLo, desc_hi,
                                           kIdescSh, kk > 0);
                            }
                        }
                        __syncwarp();
                        // Lower half (keys 0..63 -> columns 0..63, where P_t(g-1) lives):
                        // after PV_t(g-1) has read P.
                        if (g > 0) {
                            if (!(ok = warp_wait(smem_addr(&bars->pv_done[t]), (g - 1) & 1u, ctl, kSiteMmaK + 1 + t)))
                                break;
                            tc_fence_after();
                        }
                        if (leader) {
#pragma unroll
                            for (int kk = 0; kk < kD / 16; ++kk) {
                                const uint32_t off = (uint32_t)(kk >> 2) * kChunkLo + (uint32_t)(kk & 3) * 2;
                                umma_ss_lo(tmem + t * kBN, q_lo + off, k_lo + off, desc_hi, kIdescSh, kk > 0);
                            }
                            umma_commit(smem_addr(&bars->s_full[t]));
                            if (j == nk_item - 1) umma_commit(smem_addr(&bars->q_empty[t]));
                        }
                        __syncwarp();
                    }
                    if (!ok) break;
                    if (leader) umma_commit(smem_addr(&bars->k_empty[st]));
                    __syncwarp();
                } else {
                    if (!(ok = warp_wait(smem_addr(&bars->v_full[st]), par, ctl, kSiteMmaV))) break;
                    const uint32_t v_lo = v_lo0 + (uint32_t)st * kTileLo;
#pragma unroll
                    for (int t = 0; t < kQTiles; ++t) {
                        if (!(ok = warp_wait(smem_addr(&bars->p_full[t]), g & 1u, ctl, kSiteMmaV + 1 + t))) break;
                        tc_fence_after();
                        if (leader) {
#pragma unroll
                            for (int kk = 0; kk < kBN / 16; ++kk)
#pragma unroll
                                for (int ch = 0; ch < 2; ++ch)
                                    umma_ts_lo(tmem + kColO + t * kD + ch * kChunk, tmem + t * kBN + kk * 8,
                                               v_lo + ch * kChunkLo + kk * 128, desc_hi, kIdescO,
                                               (j > 0 || kk > 0) ? 1u : 0u);
                            umma_commit(smem_addr(&bars->pv_done[t]));
                        }
                        __syncwarp();
                    }
                    if (!ok) break;
                    if (leader) umma_commit(smem_addr(&bars->v_empty[st]));
                    __syncwarp();
                }
                if (++st == kStages) {
                    st = 0;
                    par ^= 1u;
                }
            }
        }
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
}

}  // namespace d128
