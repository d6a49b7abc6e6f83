// Attention backward for d = 64 on sm_100a (included by fa_fwd_sm100.cu inside
// namespace bfk, after the forward kernels). The reference declares the l / m
// slots for a backward pass (include/flash_attn.cuh:27-28) but has none; this
// computes, for upstream dO and the forward's logsumexp,
//
//   P = exp(scale Q K^T - lse),  dV = P^T dO,  dP = dO V^T,
//   dS = P o (dP - D) with D_i = sum_c dO_ic O_ic,
//   dK = scale dS^T Q,  dQ = scale dS K.
//
// One CTA per (slice, 128-row KV tile j); it walks the query tiles i:
//   * warp 8 (TMA): K_j and V_j once; per i, Q_i and dO_i (two stages) plus the
//     tile's 128 log2-lse and D values (bulk copies of a padded [BH, Npad] array);
//   * warp 9 (MMA, owns TMEM):
//       S^T  = K_j Q_i^T   (M=128 kv, N=128 q, K=64)      -> TMEM [0,128) or [128,256)
//                                                            (two buffers, by i % 2)
//       dP^T = V_j dO_i^T  (same shape)                    -> TMEM [256,384)
//     then, once the elementwise warps have written P^T and dS^T:
//       dQ_i  = dS K_j     (A = dS in shared memory, K-major) -> TMEM [256,320), over
//                                                            dP^T_i, which is read by then
//       dV_j += P^T dO_i   (A = bf16 P^T in TMEM, S^T columns 0..63) -> TMEM [384,448)
//       dK_j += dS^T Q_i   (A = bf16 dS^T in TMEM, S^T columns 64..127) -> TMEM [448,512)
//   * warps 0-7 (elementwise, two threads per KV row as in the forward): P^T,
//     dS^T into TMEM, dS into shared memory; after the dQ product, dQ_i goes to a
//     swizzled shared-memory stage and one thread adds it to the fp32 accumulator in
//     global memory with two TMA reduce-adds (the TMA unit does the read-modify-write;
//     rows past N are clipped by the tensor map); at the end dK_j and dV_j are
//     written as bf16.
// Pipelining: S^T of tile i+1 is computed (into the other buffer) while the
// elementwise warps work on tile i, and dP^T of tile i+1 as soon as dQ_i has been
// read out of TMEM, so the elementwise warps go from tile i's atomics straight to
// tile i+1's exponentials. MMAs issued by one thread run in order, so S^T of tile
// i+2 may overwrite the buffer that dV_i / dK_i read.
// Rows past N: Q/dO/K/V rows read as zero (TMA fill), padded lse is +inf, so
// those queries contribute nothing; KV rows past N are masked to P = 0 and
// never stored.
namespace bwd {

#ifndef BF_BWD_EW_REGS
#define BF_BWD_EW_REGS 216
#endif

// Warps 10 and 11 only complete the third warpgroup, so that setmaxnreg can move
// registers from the producer / MMA warpgroup to the elementwise warps.
constexpr int kThreadsB = 12 * 32;
constexpr int kEwRegs = BF_BWD_EW_REGS, kOtherRegs = 64;  // launch budget 384 x 168 = 64512
constexpr int kEwWarps = 8;
constexpr int kProdWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kTile = 128 * 64 * 2;  // 16 KiB bf16 [128 rows x 64]
constexpr int kOffK = 0;
constexpr int kOffV = kOffK + kTile;
constexpr int kOffQ = kOffV + kTile;           // [2 stages] Q_i
constexpr int kOffDO = kOffQ + 2 * kTile;      // [2 stages] dO_i
constexpr int kOffDS = kOffDO + 2 * kTile;     // dS [128 q x 128 kv] K-major: 2 chunks of 64 kv
constexpr int kOffVec = kOffDS + 2 * kTile;    // [2 stages] {lse2[128], D[128]} fp32
constexpr int kOffDQ = kOffVec + 2 * 1024;       // [2 stages][2 column halves] fp32 [128 q x 32]
constexpr int kOffBar = kOffDQ + 4 * kTile;
constexpr int kColST = 0, kColDPT = 256, kColDQ = 256, kColDV = 384, kColDK = 448;

struct Bars {
    uint64_t kv_full;
    uint64_t qd_full[2];
    uint64_t qd_empty[2];
    uint64_t s_full[2];   // S^T of the tile in buffer b computed
    uint64_t dp_full;     // dP^T computed
    uint64_t p_ready;     // P^T, dS^T (TMEM) and dS (smem) written, dP^T read
    uint64_t dq_done;     // dQ_i computed (and dS_i read from shared memory)
    uint64_t dq_free;     // dQ_i read out of TMEM
    uint64_t acc_done;    // every dV / dK product finished
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
};
constexpr int kSmemBytesB = kOffBar + (int)sizeof(Bars) + 1024;
static_assert(kSmemBytesB <= 227 * 1024, "shared memory");

struct BParams {
    int n;            // rows per slice
    int n_pad;        // n rounded up to 128 (row stride of lse2 / D)
    int q_tiles;      // n_pad / 128
    float scale;
    float scale_log2;
    const float* lse2;  // [BH, n_pad] lse * log2(e), +inf past n
    const float* dvec;  // [BH, n_pad] D, 0 past n
    float* dq_acc;      // [BH, n, 64] fp32, zeroed by the caller; receives dS K (unscaled)
    __nv_bfloat16* dk;  // [BH, n, 64]
    __nv_bfloat16* dv;  // [BH, n, 64]
    unsigned long long timeout_ns;
};

enum : unsigned {
    kSiteBProdKV = 0x600,
    kSiteBProdQ = 0x601,
    kSiteBMmaKV = 0x610,
    kSiteBMmaQ = 0x611,
    kSiteBMmaFree = 0x612,
    kSiteBMmaP = 0x613,
    kSiteBEwS = 0x620,
    kSiteBEwDone = 0x621,
};

__global__ void __launch_bounds__(kThreadsB, 1)
    fa_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                  const __grid_constant__ CUtensorMap tmDQ, const BParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int jt = (int)(blockIdx.x % (unsigned)p.q_tiles);  // KV tile (as many as query tiles)
    const int bh = (int)(blockIdx.x / (unsigned)p.q_tiles);

    if (threadIdx.x == 0) {
        mbar_init(smem_addr(&bars->kv_full), 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(smem_addr(&bars->qd_full[s]), 1);
            mbar_init(smem_addr(&bars->qd_empty[s]), 1);
        }
        mbar_init(smem_addr(&bars->s_full[0]), 1);
        mbar_init(smem_addr(&bars->s_full[1]), 1);
        mbar_init(smem_addr(&bars->dp_full), 1);
        mbar_init(smem_addr(&bars->p_ready), kEwWarps * 32);
        mbar_init(smem_addr(&bars->dq_done), 1);
        mbar_init(smem_addr(&bars->dq_free), kEwWarps * 32);
        mbar_init(smem_addr(&bars->acc_done), 1);
        mbar_init(smem_addr(&bars->drain), 1);
        bars->abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == kProdWarp && lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        tma_prefetch_desc(&tmDO);
        tma_prefetch_desc(&tmDQ);
    }
    if (warp == kMmaWarp) {
        tmem_alloc(smem_addr(&bars->tmem_base), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    const WaitCtl ctl{&bars->abort_flag, &g_wait_status, p.timeout_ns};
    static_assert(kEwWarps * 32 * kEwRegs + (kThreadsB - kEwWarps * 32) * kOtherRegs <= kThreadsB * 168,
                  "register split exceeds the launch budget");
    if (warp < kEwWarps)
        regs_inc<kEwRegs>();
    else
        regs_dec<kOtherRegs>();

    if (warp < kEwWarps) {
        // ------------------------------------------------------------ elementwise
        const int quarter = warp & 3;
        const int sub = warp >> 2;
        const int h = lane >> 4;                                 // q columns 64h .. 64h + 63
        const int row = quarter * 32 + sub * 16 + (lane & 15);   // KV row in the tile == TMEM lane
        const uint32_t lane_off = (uint32_t)(quarter * 32 + sub * 16) << 16;
        const uint32_t tDPT = tmem + lane_off + kColDPT;
        const bool kv_ok = jt * 128 + row < p.n;
        uint8_t* ds_smem = smem + kOffDS + (row >> 6) * kTile;  // chunk holding this KV column
        const int ds_unit = (row & 63) >> 3;
        // dQ_k (rows = queries): read it out of TMEM (which lets dP^T of tile k+1 be
        // computed there), stage it and add it to the fp32 accumulator by TMA.
        auto drain_dq = [&](int k) -> bool {
            if (!(warp_wait(smem_addr(&bars->dq_done), (uint32_t)k & 1u, ctl, kSiteBEwDone))) return false;
            tc_fence_after();
            {
                uint32_t o[32];
                tmem_ld16x32bx2_x32<32>(tmem + lane_off + kColDQ, o);
                tmem_wait_ld();
                tc_fence_before();
                mbar_arrive(smem_addr(&bars->dq_free));  // dP^T of the next tile may overwrite it
                // Stage k % 2 was last read by the reduce of tile k - 2.
                if (threadIdx.x == 0) tma_store_wait_read1();
                named_bar_sync(1, kEwWarps * 32);
                uint8_t* stage = smem + kOffDQ + (k & 1) * 2 * kTile + h * kTile;
#pragma unroll
                for (int c = 0; c < 8; ++c)  // 16-byte chunk c of the row at c ^ (row % 8): 128-byte swizzle
                    *reinterpret_cast<uint4*>(stage + row * 128 + ((c ^ (row & 7)) << 4)) =
                        make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
                fence_proxy_async_smem();
                named_bar_sync(1, kEwWarps * 32);
                if (threadIdx.x == 0) {
                    const uint32_t st0 = smem_addr(smem + kOffDQ + (k & 1) * 2 * kTile);
                    tma_reduce_add_3d(&tmDQ, st0, 0, k * 128, bh);
                    tma_reduce_add_3d(&tmDQ, st0 + kTile, 32, k * 128, bh);
                    tma_store_commit();
                }
            }
            return true;
        };
        bool ok = true;
        for (int i = 0; i < p.q_tiles && ok; ++i) {
            const uint32_t tST = tmem + lane_off + kColST + (uint32_t)(i & 1) * 128;
            if (!(ok = warp_wait(smem_addr(&bars->s_full[i & 1]), (uint32_t)(i >> 1) & 1u, ctl, kSiteBEwS))) break;
            tc_fence_after();
            const float* vec = reinterpret_cast<const float*>(smem + kOffVec + (i & 1) * 1024);
            const float* lse2 = vec + h * 64;
            const float* dd = vec + 128 + h * 64;

            uint32_t pk[32];  // bf16 P^T of this thread's 64 queries (pairs)
            {
                uint32_t s[2][32];
                tmem_ld16x32bx2_x32<64>(tST + 0, s[0]);
                tmem_ld16x32bx2_x32<64>(tST + 32, s[1]);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const float a = fast_exp2(__uint_as_float(s[c >> 4][(2 * c) & 31]) * p.scale_log2 - lse2[2 * c]);
                    const float b = fast_exp2(__uint_as_float(s[c >> 4][(2 * c + 1) & 31]) * p.scale_log2 - lse2[2 * c + 1]);
                    pk[c] = kv_ok ? pack_bf16x2(a, b) : 0u;
                }
            }
            // S^T has been read in full: P^T goes to its columns [0, 64), dS^T to [64, 128).
            tmem_st16x32bx2_x16<32>(tST, pk);
            tmem_st16x32bx2_x16<32>(tST + 16, pk + 16);

            // dQ of the previous tile: its product ran while this tile's P was computed.
            if (i > 0 && !(ok = drain_dq(i - 1))) break;

            // dS = P (dP - D), from the bf16 P the dV product uses (dS is rounded to bf16 too).
            if (!(ok = warp_wait(smem_addr(&bars->dp_full), (uint32_t)i & 1u, ctl, kSiteBEwS))) break;
            tc_fence_after();
            uint32_t dsk[32];
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                uint32_t dp[32];
                tmem_ld16x32bx2_x32<64>(tDPT + 32 * half, dp);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    const int q0 = half * 32 + 2 * c;
                    const uint32_t pp = pk[half * 16 + c];
                    const float p0 = __uint_as_float(pp << 16), p1 = __uint_as_float(pp & 0xffff0000u);
                    const float d0 = p0 * (__uint_as_float(dp[2 * c]) - dd[q0]);
                    const float d1 = p1 * (__uint_as_float(dp[2 * c + 1]) - dd[q0 + 1]);
                    dsk[half * 16 + c] = pack_bf16x2(d0, d1);
                }
                tmem_st16x32bx2_x16<32>(tST + 64 + 16 * half, dsk + 16 * half);
            }
            // dS [q][kv] into shared memory, 128-byte swizzled K-major rows (A of dQ = dS K).
            // Earlier readers of this buffer (dQ(i-1) = dS(i-1) K) completed before this
            // thread observed dq_done(i-1) in drain_dq(i - 1).
            // Lanes 2k and 2k+1 hold KV rows r and r+1 (r even): a 2x2 exchange gives the
            // even lane query 2c and the odd lane query 2c+1 of both rows, one 4-byte store each.
            {
                const bool odd = lane & 1;
                const int q_sub = (row & 6) * 2;  // byte offset of the row pair inside its 16-byte unit
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const uint32_t other = __shfl_xor_sync(0xffffffffu, dsk[c], 1);
                    const uint32_t v = odd ? __byte_perm(other, dsk[c], 0x7632) : __byte_perm(dsk[c], other, 0x5410);
                    const int q = h * 64 + 2 * c + (odd ? 1 : 0);
                    *reinterpret_cast<uint32_t*>(ds_smem + q * 128 + ((ds_unit ^ (q & 7)) << 4) + q_sub) = v;
                }
            }
            fence_proxy_async_smem();
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(smem_addr(&bars->p_ready));

        }
        if (ok) ok = drain_dq(p.q_tiles - 1);
        if (threadIdx.x == 0) tma_store_wait0();  // the dQ reduces have completed
        if (ok) ok = warp_wait(smem_addr(&bars->acc_done), 0u, ctl, kSiteBEwDone);
        if (ok) {
            tc_fence_after();
            // dV_j and dK_j.
            const int kv_abs = jt * 128 + row;
#pragma unroll 1
            for (int which = 0; which < 2; ++which) {
                uint32_t o[32];
                tmem_ld16x32bx2_x32<32>(tmem + lane_off + (which ? kColDK : kColDV), o);
                tmem_wait_ld();
                if (kv_ok) {
                    const float f = which ? p.scale : 1.f;
                    uint4* dst = reinterpret_cast<uint4*>((which ? p.dk : p.dv) + ((size_t)bh * p.n + kv_abs) * 64 + h * 32);
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint32_t* src = &o[c * 8];
                        uint4 v;
                        v.x = pack_bf16x2(__uint_as_float(src[0]) * f, __uint_as_float(src[1]) * f);
                        v.y = pack_bf16x2(__uint_as_float(src[2]) * f, __uint_as_float(src[3]) * f);
                        v.z = pack_bf16x2(__uint_as_float(src[4]) * f, __uint_as_float(src[5]) * f);
                        v.w = pack_bf16x2(__uint_as_float(src[6]) * f, __uint_as_float(src[7]) * f);
                        dst[c] = v;
                    }
                }
            }
        }
    } else if (warp == kProdWarp) {
        // ------------------------------------------------------------ TMA producer
        const bool leader = elect_one();
        const uint32_t kvf = smem_addr(&bars->kv_full);
        if (leader) {
            mbar_arrive_expect_tx(kvf, 2 * kTile);
            tma_load_3d(smem_addr(smem + kOffK), &tmK, kvf, 0, jt * 128, bh);
            tma_load_3d(smem_addr(smem + kOffV), &tmV, kvf, 0, jt * 128, bh);
        }
        __syncwarp();
        bool ok = true;
        int last = -1;
        for (int i = 0; i < p.q_tiles && ok; ++i) {
            const int s = i & 1;
            if (!(ok = warp_wait(smem_addr(&bars->qd_empty[s]), (uint32_t)((i >> 1) & 1) ^ 1u, ctl, kSiteBProdQ))) break;
            if (leader) {
                const uint32_t f = smem_addr(&bars->qd_full[s]);
                mbar_arrive_expect_tx(f, 2 * kTile + 1024);
                tma_load_3d(smem_addr(smem + kOffQ + s * kTile), &tmQ, f, 0, i * 128, bh);
                tma_load_3d(smem_addr(smem + kOffDO + s * kTile), &tmDO, f, 0, i * 128, bh);
                const size_t off = (size_t)bh * p.n_pad + (size_t)i * 128;
                bulk_load(smem_addr(smem + kOffVec + s * 1024), p.lse2 + off, 512, f);
                bulk_load(smem_addr(smem + kOffVec + s * 1024 + 512), p.dvec + off, 512, f);
            }
            last = i;
            __syncwarp();
        }
        if (*ctl.abort_flag) {
            int never = 0;
            const WaitCtl drain{&never, nullptr, ctl.limit_ns};
            mbar_wait(kvf, 0u, drain, 0);
            if (last >= 0) mbar_wait(smem_addr(&bars->qd_full[last & 1]), (uint32_t)(last >> 1) & 1u, drain, 0);
            if (last >= 1)
                mbar_wait(smem_addr(&bars->qd_full[(last - 1) & 1]), (uint32_t)((last - 1) >> 1) & 1u, drain, 0);
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------------ MMA issuer
        constexpr uint32_t kIdescT = idesc_bf16_f32(128, 128, 0);  // K-major x K-major, N = 128 queries
        constexpr uint32_t kIdescG = idesc_bf16_f32(128, 64, 1);   // A x (MN-major, N = 64 head dims)
        const bool leader = elect_one();
        const uint64_t desc_base = smem_desc_sw128(smem_addr(smem), 16, 1024);
        const uint32_t desc_hi = (uint32_t)(desc_base >> 32);
        const uint32_t lo0 = (uint32_t)desc_base;
        constexpr uint32_t kTileLo = kTile >> 4;
        const uint32_t k_lo = lo0 + (kOffK >> 4), v_lo = lo0 + (kOffV >> 4), ds_lo = lo0 + (kOffDS >> 4);
        bool ok = warp_wait(smem_addr(&bars->kv_full), 0u, ctl, kSiteBMmaKV);
        tc_fence_after();
        const int T = p.q_tiles;
        auto q_lo = [&](int i) { return lo0 + ((kOffQ >> 4) + (uint32_t)(i & 1) * kTileLo); };
        auto do_lo = [&](int i) { return lo0 + ((kOffDO >> 4) + (uint32_t)(i & 1) * kTileLo); };
        auto wait_qd = [&](int i) {
            const bool r = warp_wait(smem_addr(&bars->qd_full[i & 1]), (uint32_t)(i >> 1) & 1u, ctl, kSiteBMmaQ);
            tc_fence_after();
            return r;
        };
        auto issue_st = [&](int i) {  // S^T_i = K Q_i^T into buffer i % 2
            if (leader) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_ss_lo(tmem + kColST + (uint32_t)(i & 1) * 128, k_lo + kk * 2, q_lo(i) + kk * 2, desc_hi, kIdescT,
                               kk > 0);
                umma_commit(smem_addr(&bars->s_full[i & 1]));
            }
            __syncwarp();
        };
        auto issue_dpt = [&](int i) {  // dP^T_i = V dO_i^T
            if (leader) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_ss_lo(tmem + kColDPT, v_lo + kk * 2, do_lo(i) + kk * 2, desc_hi, kIdescT, kk > 0);
                umma_commit(smem_addr(&bars->dp_full));
            }
            __syncwarp();
        };
        if (ok && (ok = wait_qd(0))) {
            issue_st(0);
            issue_dpt(0);
            if (T > 1 && (ok = wait_qd(1))) issue_st(1);
        }
        for (int i = 0; i < T && ok; ++i) {
            if (!(ok = warp_wait(smem_addr(&bars->p_ready), (uint32_t)i & 1u, ctl, kSiteBMmaP))) break;
            tc_fence_after();
            const uint32_t st_col = tmem + kColST + (uint32_t)(i & 1) * 128;
            if (leader) {
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)  // 16 KV rows per step: dS chunk (kk / 4), K rows 16 kk
                    umma_ss_lo(tmem + kColDQ, ds_lo + (uint32_t)(kk >> 2) * kTileLo + (uint32_t)(kk & 3) * 2,
                               k_lo + kk * 128, desc_hi, kIdescG, kk > 0);
                umma_commit(smem_addr(&bars->dq_done));
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)  // 16 queries per step: 8 TMEM columns of P^T, 16 x 128 B of dO
                    umma_ts_lo(tmem + kColDV, st_col + kk * 8, do_lo(i) + kk * 128, desc_hi, kIdescG,
                               (i > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    umma_ts_lo(tmem + kColDK, st_col + 64 + kk * 8, q_lo(i) + kk * 128, desc_hi, kIdescG,
                               (i > 0 || kk > 0) ? 1u : 0u);
                umma_commit(smem_addr(&bars->qd_empty[i & 1]));
                if (i == T - 1) umma_commit(smem_addr(&bars->acc_done));
            }
            __syncwarp();
            if (i + 1 < T) {
                if (!(ok = warp_wait(smem_addr(&bars->dq_free), (uint32_t)i & 1u, ctl, kSiteBMmaFree))) break;
                tc_fence_after();
                issue_dpt(i + 1);
            }
            if (i + 2 < T) {
                if (!(ok = wait_qd(i + 2))) break;
                issue_st(i + 2);
            }
        }
        if (leader) umma_commit(smem_addr(&bars->drain));
        __syncwarp();
        int never = 0;
        const WaitCtl drain{&never, nullptr, ctl.limit_ns};
        mbar_wait(smem_addr(&bars->drain), 0u, drain, 0);
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// D_r = sum_c dO_rc O_rc and lse2_r = lse_r log2(e) over [BH, n_pad]; padded rows get
// D = 0 and lse2 = +inf (so exp2(s - lse2) = 0 for them). One warp per row.
__global__ void bwd_prep_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                const float* __restrict__ lse, float* __restrict__ dvec, float* __restrict__ lse2,
                                long long bh, int n, int n_pad) {
    const long long rows = bh * n_pad;
    const int lane = threadIdx.x & 31;
    for (long long r = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows;
         r += ((long long)gridDim.x * blockDim.x) >> 5) {
        const long long s = r / n_pad;
        const int i = (int)(r - s * n_pad);
        float acc = 0.f;
        if (i < n) {
            const size_t base = ((size_t)s * n + i) * 64 + lane * 2;
            const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(o + base);
            const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(dout + base);
            acc = __bfloat162float(a.x) * __bfloat162float(b.x) + __bfloat162float(a.y) * __bfloat162float(b.y);
        }
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
        if (lane == 0) {
            dvec[r] = acc;
            lse2[r] = i < n ? lse[(size_t)s * n + i] * 1.4426950408889634f : INFINITY;
        }
    }
}

// dQ = scale * dq_acc, to bf16.
__global__ void bwd_dq_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq, float scale, size_t count4) {
    for (size_t k = (size_t)blockIdx.x * blockDim.x + threadIdx.x; k < count4; k += (size_t)gridDim.x * blockDim.x) {
        const float4 a = reinterpret_cast<const float4*>(acc)[k];
        uint2 v;
        v.x = pack_bf16x2(a.x * scale, a.y * scale);
        v.y = pack_bf16x2(a.z * scale, a.w * scale);
        reinterpret_cast<uint2*>(dq)[k] = v;
    }
}

}  // namespace bwd
