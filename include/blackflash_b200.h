/*
 * BlackFlash-B200 C ABI: attention forward (non-causal, bf16, head dim 64, or 128 as an extension) on
 * sm_100a.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t passed
 * as `void*`. Calls are asynchronous on that stream. They return BF_OK or an
 * error code, and blackflash_last_error() gives the message for the calling
 * thread. No entry point allocates device memory or synchronises the device,
 * except blackflash_ring_create / blackflash_ring_destroy (which own the ring's
 * buffers) and the ones documented as synchronous (the status reads).
 *
 * Layouts: Q, K, V and O are contiguous [B, H, N, d] bf16, d = 64 or 128 (the same layout as
 * the reference, binding/blackflash_ops.cu:24-27). lse and row_max are [B, H, N]
 * fp32.
 */
#ifndef BLACKFLASH_B200_H
#define BLACKFLASH_B200_H

#ifdef __cplusplus
extern "C" {
#endif

#define BF_OK 0
#define BF_ERR_ARG 1     /* bad shape, pointer or alignment */
#define BF_ERR_CUDA 2    /* a CUDA runtime/driver call failed */
#define BF_ERR_TIMEOUT 3 /* a device-side wait exceeded its limit (see blackflash_status) */

/*
 * O = softmax(scale * Q K^T) V for every (b, h) slice.
 *
 * Replaces flash_attn_naive_launch (reference include/flash_attn.cuh:22-32,
 * kernel/flash_attn_mma.cu:470-518). The arguments mean the same, with three
 * differences: it returns a status instead of calling exit(), it takes the
 * stream as void*, and it fills `lse` / `row_max` when they are non-null.
 * The reference documents those two slots but never writes them.
 *   lse[b,h,i]     = log(sum_j exp(scale * S_ij))   (natural log)
 *   row_max[b,h,i] = max_j scale * S_ij
 * Requirements: d == 64 (reference) or 128 (blackflash_fwd, blackflash_fwd_causal), B, H, N >= 1, every pointer 16-byte aligned.
 * N need not be a multiple of 128: the kernel masks the ragged KV tile and
 * skips stores past row N.
 */
int blackflash_fwd(const void* Q, const void* K, const void* V, void* O, float* lse, float* row_max, int B, int H,
                   int N, int d, float scale, void* stream);

/*
 * blackflash_fwd with a causal mask: query i attends to keys j <= i (top-left
 * aligned, Q and K of the same length N). Tiles above the diagonal are skipped,
 * so the work is about half. lse / row_max are taken over the visible keys. No
 * counterpart in the reference kernel (non-causal only); its benchmark times the
 * causal case with cuDNN (tests/bench_blackflash.py:58-60).
 */
int blackflash_fwd_causal(const void* Q, const void* K, const void* V, void* O, float* lse, float* row_max, int B,
                          int H, int N, int d, float scale, void* stream);

/*
 * Partial attention of one query block against one KV block. It is the
 * per-step kernel of the ring (sequence-parallel) mode and has no counterpart
 * in the reference.
 *   Q: [BH, Nq, 64] bf16; K, V: [BH, Nkv, 64] bf16
 *   O_f32: [BH, Nq, 64] fp32, normalised over this KV block only
 *   lse:   [BH, Nq] fp32 logsumexp over this KV block (required)
 */
int blackflash_fwd_partial(const void* Q, const void* K, const void* V, float* O_f32, float* lse, long long BH,
                           int Nq, int Nkv, int d, float scale, void* stream);

/*
 * Partial attention of one query block against gathered KV blocks: the
 * sequence-parallel mode's second kernel, after an all-gather of K and V.
 * No counterpart in the reference.
 *   Q:      [BH, Nq, 64] bf16
 *   Kg, Vg: [n_blocks, BH, block_rows, 64] bf16 (rank-major, as an all-gather lays it out)
 *   skip:   block left out (the caller's own, already computed), or -1 to use all
 *   O_f32, lse as in blackflash_fwd_partial, over the concatenation of the used
 *   blocks. block_rows must be a multiple of 128.
 */
int blackflash_fwd_partial_blocks(const void* Q, const void* Kg, const void* Vg, float* O_f32, float* lse,
                                  long long BH, int Nq, int n_blocks, int block_rows, int skip, int d, float scale,
                                  void* stream);

/*
 * Attention backward (d = 64). No counterpart in the reference: its l / m slots
 * (include/flash_attn.cuh:27-28) are declared for a backward pass it never built.
 *   Q, K, V, O, dO: [B, H, N, 64] bf16 (O from the forward), lse: [B, H, N] fp32 from
 *   blackflash_fwd's lse slot; dQ, dK, dV: [B, H, N, 64] bf16 outputs.
 *   workspace: caller-owned device memory of at least
 *   blackflash_bwd_workspace_bytes(B, H, N, 64) bytes (fp32 dQ accumulator and two
 *   [B, H, N rounded up to 128] fp32 vectors); it is overwritten.
 * Asynchronous on `stream`; three kernels and one memset.
 */
long long blackflash_bwd_workspace_bytes(int B, int H, int N, int d);
int blackflash_bwd(const void* Q, const void* K, const void* V, const void* O, const void* dO, const float* lse,
                   void* dQ, void* dK, void* dV, void* workspace, long long workspace_bytes, int B, int H, int N,
                   int d, float scale, void* stream);

/*
 * The backward without a workspace argument, for callers that cannot allocate
 * device memory: plugins whose host owns the whole device pool, or loops that
 * cannot afford the synchronisation cudaMalloc / cudaFree may bring. No
 * counterpart in the reference. It allocates nothing; its scratch is a fixed
 * 64 MiB array inside the library on every device that loads it, so
 * B * H * N is limited to about 250000 rows (larger problems get BF_ERR_ARG and
 * belong to blackflash_bwd). The first call on a device looks up the array's
 * device address; make it before any stream capture. That address is kept until
 * the process exits, so do not call this again on a device after cudaDeviceReset.
 * All calls on a device share
 * the array: calls in order on one stream are fine, calls that overlap on the
 * GPU race. Arguments as blackflash_bwd.
 */
int blackflash_bwd_noalloc(const void* Q, const void* K, const void* V, const void* O, const void* dO,
                           const float* lse, void* dQ, void* dK, void* dV, int B, int H, int N, int d, float scale,
                           void* stream);

/*
 * Log-sum-exp merge of one partial result into a running one, in place:
 *   lse' = log(exp(lse_acc) + exp(lse_part))
 *   O'   = O_acc * exp(lse_acc - lse') + O_part * exp(lse_part - lse')
 * rows = BH * Nq. A row whose lse_acc is -inf takes the partial unchanged.
 */
int blackflash_lse_merge(float* O_acc, float* lse_acc, const float* O_part, const float* lse_part, long long rows,
                         int d, void* stream);

/* fp32 -> bf16 (round to nearest even), n elements. */
int blackflash_f32_to_bf16(const float* src, void* dst, long long n, void* stream);

/*
 * Sequence-parallel forward over G processes (one per GPU of a node), KV blocks
 * moved round the ring in both directions by peer copies into the neighbours'
 * memory (CUDA IPC, copy engines over NVLink) and merged by log-sum-exp. The
 * schedule of the NCCL ring in blackflash_b200/ring.py, driven from C++ with
 * GPU-side flags; no counterpart in the reference, which has no multi-GPU mode.
 *   1. blackflash_ring_create(world, rank, BH, n, 64, &ring, handle): allocates
 *      the ring's buffers on the current device (two receive slots of two K and
 *      two V blocks, fp32 accumulators) and writes this rank's IPC handle
 *      (blackflash_ring_handle_bytes() bytes). n: rows per rank, a multiple of 128.
 *   2. Exchange the handles (all ranks' handles, concatenated in rank order) and
 *      call blackflash_ring_connect(ring, handles).
 *   3. blackflash_ring_forward(ring, Q, K, V, O, lse, scale, stream), collectively:
 *      Q, K, V [BH, n, 64] bf16 are this rank's rows; O [BH, n, 64] bf16 and lse
 *      [BH, n] fp32 (optional) receive this rank's rows of the full attention.
 *      Asynchronous on `stream`; K and V must stay unchanged until it completes.
 *   blackflash_ring_status reads (and optionally clears) the ring's wait-timeout
 *   word: a wait on a neighbour that gave up after 10 s gives BF_ERR_TIMEOUT.
 *   blackflash_ring_destroy synchronises the device and frees everything.
 */
int blackflash_ring_handle_bytes(void);
int blackflash_ring_create(int world, int rank, long long BH, int n, int d, void** ring, void* handle_out);
int blackflash_ring_connect(void* ring, const void* handles);
int blackflash_ring_forward(void* ring, const void* Q, const void* K, const void* V, void* O, float* lse, float scale,
                            void* stream);
int blackflash_ring_status(void* ring, int reset, unsigned* out);
int blackflash_ring_destroy(void* ring);

/*
 * Wait-timeout status of the current device. It is synchronous: it reads a
 * device word that a kernel sets when one of its bounded mbarrier waits gives
 * up. *out receives 0 if no wait gave up, otherwise the code of the first wait
 * site that did. With reset != 0 the word is cleared after it is read.
 */
int blackflash_status(int reset, unsigned* out);

/* Message for the last error returned on this thread ("" if none). */
const char* blackflash_last_error(void);

/* ABI version of this library (incremented on any signature change). */
int blackflash_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* BLACKFLASH_B200_H */
