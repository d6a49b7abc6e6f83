// Sequence-parallel attention forward with the KV blocks moved round the ring by
// the copy engines over NVLink (CUDA IPC peer copies) instead of NCCL send/recv.
// No counterpart in the reference (it has no multi-GPU mode); the schedule is the
// both-way ring of blackflash_b200/ring.py (_ring_bidirectional), driven from C++.
//
// Rank r of G holds rows [r n, (r + 1) n) of Q, K and V for all BH slices. At step
// s >= 1 it computes L_s = block r - s and (for s <= nr) R_s = block r + s, with
// nl = floor(G / 2) steps in all and nr = ceil(G / 2) - 1, so each foreign block
// is computed once. L_{s+1} is the left neighbour's L_s, pushed by that neighbour
// into this rank's receive slot; R_{s+1} likewise comes from the right. The
// receive buffer of every rank is exported with cudaIpcGetMemHandle and opened by
// its two neighbours, so a transfer is one cudaMemcpyAsync per tensor straight
// into the neighbour's local HBM: no SM time, no library kernel reading peer
// memory, no multicast. Kernels only ever read local memory.
//
// Synchronisation is GPU-side, through 32-bit flags in each rank's exported
// buffer: a one-thread kernel stores a step stamp into a neighbour's flag after a
// copy (arrival) or after this rank is done with a slot (slot free); a one-thread
// kernel waits for a local flag with a bounded spin (timeout -> status word and
// BF_ERR_TIMEOUT from blackflash_ring_status, never a hang). Stamps grow
// monotonically, epoch * 64 + step, so flags are never reset between calls.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <new>

#include "fa_fwd_sm100.h"

namespace {

constexpr int kFlagArrL = 0;   // written by the left neighbour: L slot of step (stamp) filled
constexpr int kFlagArrR = 1;   // written by the right neighbour: R slot filled
constexpr int kFlagFreeL = 2;  // written by the right neighbour: its L slot of step (stamp) free
constexpr int kFlagFreeR = 3;  // written by the left neighbour: its R slot free
constexpr int kFlagErr = 8;    // set by a wait that gave up
constexpr size_t kFlagBytes = 4096;
constexpr unsigned kEpochStride = 64;

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits (one thread, bounded) until *flag >= target; on timeout records `site` in
// err (first writer wins) and returns, leaving the stream to run on.
__global__ void flag_wait_kernel(const unsigned* flag, unsigned target, unsigned long long timeout_ns, unsigned* err,
                                 unsigned site) {
    const uint64_t t0 = now_ns();
    while (ld_acquire_sys(flag) < target) {
        if (now_ns() - t0 > timeout_ns) {
            atomicCAS(err, 0u, site);
            return;
        }
        __nanosleep(200);
    }
}

__global__ void flag_set_kernel(unsigned* flag, unsigned value) {
    __threadfence_system();
    st_release_sys(flag, value);
}

}  // namespace

struct BfRing {
    int world, rank, dev;
    long long bh;
    int n, d;
    size_t blk;             // bytes of one K (or V) block
    unsigned epoch;
    unsigned long long timeout_ns;
    unsigned char* buf;     // [flags | slot 0: K pair, V pair | slot 1: K pair, V pair]
    unsigned char* left_buf;   // the neighbours' buffers, opened through IPC
    unsigned char* right_buf;
    float *o_acc, *o_part, *lse_part, *lse_tmp;
    cudaStream_t s_l, s_r, s_sig;
    cudaEvent_t ev_start, ev_l[33], ev_r[33], ev_c[33], ev_end_l, ev_end_r, ev_end_sig;
};

namespace {

unsigned* flags(unsigned char* base) { return reinterpret_cast<unsigned*>(base); }
// Slot s (1 or 0), pair index (0 = L, 1 = R), tensor (0 = K, 1 = V).
unsigned char* slot_ptr(const BfRing* r, unsigned char* base, int slot, int t, int pair) {
    return base + kFlagBytes + ((size_t)slot * 4 + (size_t)t * 2 + pair) * r->blk;
}

int cuda_err(cudaError_t e, const char* what) {
    char msg[256];
    snprintf(msg, sizeof(msg), "%s: %s", what, cudaGetErrorString(e));
    return bf_set_error(BF_ERR_CUDA, msg);
}
#define RCK(call, what)                                    \
    do {                                                   \
        cudaError_t e_ = (call);                           \
        if (e_ != cudaSuccess) return cuda_err(e_, what);  \
    } while (0)

int wait_flag(BfRing* r, cudaStream_t st, int idx, unsigned target, unsigned site) {
    flag_wait_kernel<<<1, 1, 0, st>>>(flags(r->buf) + idx, target, r->timeout_ns, flags(r->buf) + kFlagErr, site);
    RCK(cudaGetLastError(), "ring flag wait");
    return BF_OK;
}

int set_flag(unsigned char* peer_base, int idx, unsigned value, cudaStream_t st) {
    flag_set_kernel<<<1, 1, 0, st>>>(flags(peer_base) + idx, value);
    RCK(cudaGetLastError(), "ring flag set");
    return BF_OK;
}

}  // namespace

extern "C" int blackflash_ring_destroy(void* ring);

extern "C" int blackflash_ring_create(int world, int rank, long long BH, int n, int d, void** ring, void* handle_out) {
    bf_set_error(BF_OK, "");
    if (!ring || !handle_out) return bf_set_error(BF_ERR_ARG, "null ring or handle pointer");
    if (world < 2 || world > 64 || rank < 0 || rank >= world)
        return bf_set_error(BF_ERR_ARG, "ring needs 2 <= world <= 64 and 0 <= rank < world");
    if (BH <= 0 || n <= 0 || n % 128 || d != 64)
        return bf_set_error(BF_ERR_ARG, "ring needs d = 64, BH >= 1 and a per-rank block of a multiple of 128 rows");
    BfRing* r = new (std::nothrow) BfRing();
    if (!r) return bf_set_error(BF_ERR_ARG, "out of host memory");
    r->world = world;
    r->rank = rank;
    r->bh = BH;
    r->n = n;
    r->d = d;
    r->blk = (size_t)BH * n * d * 2;
    r->epoch = 0;
    r->timeout_ns = 10000000000ull;
    auto fail = [&](int rc) {
        delete r;
        return rc;
    };
    if (cudaGetDevice(&r->dev) != cudaSuccess) return fail(bf_set_error(BF_ERR_CUDA, "cudaGetDevice failed"));
    cudaError_t e = cudaMalloc(&r->buf, kFlagBytes + 8 * r->blk);
    if (e != cudaSuccess) return fail(cuda_err(e, "ring buffer"));
    // Flags start at the end stamp of "epoch 0", so the first call finds every slot free.
    unsigned init[kFlagBytes / 4];
    memset(init, 0, sizeof(init));
    init[kFlagFreeL] = init[kFlagFreeR] = kEpochStride - 1;
    e = cudaMemcpy(r->buf, init, sizeof(init), cudaMemcpyHostToDevice);
    const size_t f32 = (size_t)BH * n * d * 4;
    if (e == cudaSuccess) e = cudaMalloc(&r->o_acc, f32);
    if (e == cudaSuccess) e = cudaMalloc(&r->o_part, f32);
    if (e == cudaSuccess) e = cudaMalloc(&r->lse_part, (size_t)BH * n * 4);
    if (e == cudaSuccess) e = cudaMalloc(&r->lse_tmp, (size_t)BH * n * 4);
    for (cudaStream_t* s : {&r->s_l, &r->s_r, &r->s_sig})
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(s, cudaStreamNonBlocking);
    cudaEvent_t* evs[] = {&r->ev_start, &r->ev_end_l, &r->ev_end_r, &r->ev_end_sig};
    for (cudaEvent_t* ev : evs)
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
    for (int i = 0; i < 33 && e == cudaSuccess; ++i) {
        e = cudaEventCreateWithFlags(&r->ev_l[i], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&r->ev_r[i], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&r->ev_c[i], cudaEventDisableTiming);
    }
    if (e == cudaSuccess) {
        cudaIpcMemHandle_t h;
        e = cudaIpcGetMemHandle(&h, r->buf);
        if (e == cudaSuccess) memcpy(handle_out, &h, sizeof(h));
    }
    if (e != cudaSuccess) {
        const int rc = cuda_err(e, "ring set-up");
        void* rv = r;
        blackflash_ring_destroy(rv);
        return rc;
    }
    *ring = r;
    return BF_OK;
}

extern "C" int blackflash_ring_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

extern "C" int blackflash_ring_connect(void* ring, const void* handles) {
    bf_set_error(BF_OK, "");
    BfRing* r = static_cast<BfRing*>(ring);
    if (!r || !handles) return bf_set_error(BF_ERR_ARG, "null ring or handles");
    if (r->left_buf) return bf_set_error(BF_ERR_ARG, "ring already connected");
    const int left = (r->rank + r->world - 1) % r->world, right = (r->rank + 1) % r->world;
    const unsigned char* hb = static_cast<const unsigned char*>(handles);
    cudaIpcMemHandle_t hl, hr;
    memcpy(&hl, hb + (size_t)left * sizeof(hl), sizeof(hl));
    memcpy(&hr, hb + (size_t)right * sizeof(hr), sizeof(hr));
    void* p = nullptr;
    RCK(cudaIpcOpenMemHandle(&p, hl, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle (left)");
    r->left_buf = static_cast<unsigned char*>(p);
    if (right == left) {
        r->right_buf = r->left_buf;  // two ranks: one neighbour on both sides
    } else {
        p = nullptr;
        RCK(cudaIpcOpenMemHandle(&p, hr, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle (right)");
        r->right_buf = static_cast<unsigned char*>(p);
    }
    return BF_OK;
}

extern "C" int blackflash_ring_forward(void* ring, const void* Q, const void* K, const void* V, void* O, float* lse,
                                       float scale, void* stream) {
    bf_set_error(BF_OK, "");
    BfRing* r = static_cast<BfRing*>(ring);
    if (!r || !Q || !K || !V || !O) return bf_set_error(BF_ERR_ARG, "null pointer");
    if (!r->left_buf) return bf_set_error(BF_ERR_ARG, "ring not connected");
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != r->dev)
        return bf_set_error(BF_ERR_ARG, "ring used on another device than it was created on");
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    const int G = r->world, nl = G / 2, nr = (G + 1) / 2 - 1;
    const unsigned ep = ++r->epoch * kEpochStride;
    const unsigned prev_end = ep - 1;  // every slot was freed at the end of the previous call
    float* lse_acc = lse ? lse : r->lse_tmp;
    int rc;

    RCK(cudaEventRecord(r->ev_start, cs), "event");
    RCK(cudaStreamWaitEvent(r->s_l, r->ev_start, 0), "event wait");
    RCK(cudaStreamWaitEvent(r->s_r, r->ev_start, 0), "event wait");
    RCK(cudaStreamWaitEvent(r->s_sig, r->ev_start, 0), "event wait");

    // Pushes. Direction L: my L_s (own block at s = 0) -> right neighbour's slot (s+1)%2,
    // pair 0; direction R: my R_s -> left neighbour's slot (s+1)%2, pair 1.
    for (int dir = 0; dir < 2; ++dir) {
        const int steps = dir == 0 ? nl : nr;
        cudaStream_t st = dir == 0 ? r->s_l : r->s_r;
        unsigned char* dst_base = dir == 0 ? r->right_buf : r->left_buf;
        const int arr_flag = dir == 0 ? kFlagArrL : kFlagArrR, free_flag = dir == 0 ? kFlagFreeL : kFlagFreeR;
        for (int s = 0; s < steps; ++s) {
            const unsigned char *src_k, *src_v;
            if (s == 0) {
                src_k = static_cast<const unsigned char*>(K);
                src_v = static_cast<const unsigned char*>(V);
            } else {
                if ((rc = wait_flag(r, st, arr_flag, ep + s, 0x500u + dir)) != BF_OK) return rc;
                src_k = slot_ptr(r, r->buf, s % 2, 0, dir);
                src_v = slot_ptr(r, r->buf, s % 2, 1, dir);
            }
            // The neighbour's slot (s+1)%2 last held step s-1 of this call, or for s < 2
            // a step of the previous call.
            const unsigned free_at = s + 1 >= 3 ? ep + (s - 1) : prev_end;
            if ((rc = wait_flag(r, st, free_flag, free_at, 0x510u + dir)) != BF_OK) return rc;
            RCK(cudaMemcpyAsync(slot_ptr(r, dst_base, (s + 1) % 2, 0, dir), src_k, r->blk, cudaMemcpyDeviceToDevice, st),
                "ring peer copy");
            RCK(cudaMemcpyAsync(slot_ptr(r, dst_base, (s + 1) % 2, 1, dir), src_v, r->blk, cudaMemcpyDeviceToDevice, st),
                "ring peer copy");
            if ((rc = set_flag(dst_base, arr_flag, ep + s + 1, st)) != BF_OK) return rc;
            RCK(cudaEventRecord(dir == 0 ? r->ev_l[s] : r->ev_r[s], st), "event");
        }
        RCK(cudaEventRecord(dir == 0 ? r->ev_end_l : r->ev_end_r, st), "event");
    }

    // Compute on the caller's stream: own block, then each step's blocks, merged.
    if ((rc = blackflash_fwd_partial(Q, K, V, r->o_acc, lse_acc, r->bh, r->n, r->n, r->d, scale, cs)) != BF_OK) return rc;
    for (int s = 1; s <= nl; ++s) {
        const int slot = s % 2;
        if ((rc = wait_flag(r, cs, kFlagArrL, ep + s, 0x520u)) != BF_OK) return rc;
        if (s <= nr) {
            if ((rc = wait_flag(r, cs, kFlagArrR, ep + s, 0x521u)) != BF_OK) return rc;
            rc = blackflash_fwd_partial_blocks(Q, slot_ptr(r, r->buf, slot, 0, 0), slot_ptr(r, r->buf, slot, 1, 0),
                                               r->o_part, r->lse_part, r->bh, r->n, 2, r->n, -1, r->d, scale, cs);
        } else {
            rc = blackflash_fwd_partial(Q, slot_ptr(r, r->buf, slot, 0, 0), slot_ptr(r, r->buf, slot, 1, 0), r->o_part,
                                        r->lse_part, r->bh, r->n, r->n, r->d, scale, cs);
        }
        if (rc != BF_OK) return rc;
        if ((rc = blackflash_lse_merge(r->o_acc, lse_acc, r->o_part, r->lse_part, r->bh * r->n, r->d, cs)) != BF_OK)
            return rc;
        RCK(cudaEventRecord(r->ev_c[s], cs), "event");
        // Slot s%2 is free once this step's kernels and this rank's forwarding copies
        // out of it are done: tell the neighbours that write into it.
        RCK(cudaStreamWaitEvent(r->s_sig, r->ev_c[s], 0), "event wait");
        if (s < nl) RCK(cudaStreamWaitEvent(r->s_sig, r->ev_l[s], 0), "event wait");
        if (s < nr) RCK(cudaStreamWaitEvent(r->s_sig, r->ev_r[s], 0), "event wait");
        if ((rc = set_flag(r->left_buf, kFlagFreeL, ep + s, r->s_sig)) != BF_OK) return rc;
        if (s <= nr && (rc = set_flag(r->right_buf, kFlagFreeR, ep + s, r->s_sig)) != BF_OK) return rc;
    }
    // Every slot is free for the next call once all of this call's steps and copies are done.
    RCK(cudaStreamWaitEvent(r->s_sig, r->ev_end_l, 0), "event wait");
    RCK(cudaStreamWaitEvent(r->s_sig, r->ev_end_r, 0), "event wait");
    RCK(cudaStreamWaitEvent(r->s_sig, r->ev_c[nl], 0), "event wait");
    if ((rc = set_flag(r->left_buf, kFlagFreeL, ep + kEpochStride - 1, r->s_sig)) != BF_OK) return rc;
    if ((rc = set_flag(r->right_buf, kFlagFreeR, ep + kEpochStride - 1, r->s_sig)) != BF_OK) return rc;
    RCK(cudaEventRecord(r->ev_end_sig, r->s_sig), "event");

    if ((rc = blackflash_f32_to_bf16(r->o_acc, O, r->bh * r->n * r->d, cs)) != BF_OK) return rc;
    // The caller's stream does not run on until the pushes of its K / V have finished.
    RCK(cudaStreamWaitEvent(cs, r->ev_end_l, 0), "event wait");
    RCK(cudaStreamWaitEvent(cs, r->ev_end_r, 0), "event wait");
    RCK(cudaStreamWaitEvent(cs, r->ev_end_sig, 0), "event wait");
    return BF_OK;
}

extern "C" int blackflash_ring_status(void* ring, int reset, unsigned* out) {
    BfRing* r = static_cast<BfRing*>(ring);
    if (!r) return bf_set_error(BF_ERR_ARG, "null ring");
    unsigned v = 0;
    RCK(cudaMemcpy(&v, flags(r->buf) + kFlagErr, 4, cudaMemcpyDeviceToHost), "ring status");
    if (reset) RCK(cudaMemset(flags(r->buf) + kFlagErr, 0, 4), "ring status reset");
    if (out) *out = v;
    return v ? bf_set_error(BF_ERR_TIMEOUT, "a ring wait gave up (a neighbour stopped or is too slow)") : BF_OK;
}

extern "C" int blackflash_ring_destroy(void* ring) {
    BfRing* r = static_cast<BfRing*>(ring);
    if (!r) return BF_OK;
    cudaDeviceSynchronize();
    if (r->left_buf) cudaIpcCloseMemHandle(r->left_buf);
    if (r->right_buf && r->right_buf != r->left_buf) cudaIpcCloseMemHandle(r->right_buf);
    for (cudaStream_t s : {r->s_l, r->s_r, r->s_sig})
        if (s) cudaStreamDestroy(s);
    for (cudaEvent_t ev : {r->ev_start, r->ev_end_l, r->ev_end_r, r->ev_end_sig})
        if (ev) cudaEventDestroy(ev);
    for (int i = 0; i < 33; ++i)
        for (cudaEvent_t ev : {r->ev_l[i], r->ev_r[i], r->ev_c[i]})
            if (ev) cudaEventDestroy(ev);
    for (void* p : {(void*)r->buf, (void*)r->o_acc, (void*)r->o_part, (void*)r->lse_part, (void*)r->lse_tmp})
        if (p) cudaFree(p);
    delete r;
    return BF_OK;
}
