// C-ABI entry points (include/blackflash_b200.h, test hooks in
// include/blackflash_b200_diag.h) and the C++ launcher with the
// reference's signature (include/flash_attn.cuh). All argument checking that
// does not need the device lives in bf_fwd_launch (fa_fwd_sm100.cu).
#include <stdio.h>
#include <string.h>

#include "../../include/flash_attn.cuh"
#include "fa_fwd_sm100.h"

namespace {
thread_local char g_last_error[512] = {0};
}

int bf_set_error(int code, const char* msg) {
    snprintf(g_last_error, sizeof(g_last_error), "%s", msg ? msg : "");
    return code;
}

extern "C" const char* blackflash_last_error(void) { return g_last_error; }

extern "C" int blackflash_abi_version(void) { return 1; }

static BfFwdArgs base_args(const void* Q, const void* K, const void* V, int B, int H, int N, int d, float scale,
                           void* stream) {
    BfFwdArgs a;
    memset(&a, 0, sizeof(a));
    a.q = Q;
    a.k = K;
    a.v = V;
    a.bh = (long long)B * (long long)H;
    a.n_q = N;
    a.n_kv = N;
    a.d = d;
    a.scale = scale;
    a.stream = stream;
    return a;
}

static int check_bhn(int B, int H, int N) {
    if (B <= 0 || H <= 0 || N <= 0) return bf_set_error(BF_ERR_ARG, "empty problem: B, H and N must be >= 1");
    return BF_OK;
}

extern "C" int blackflash_fwd(const void* Q, const void* K, const void* V, void* O, float* lse, float* row_max, int B,
                              int H, int N, int d, float scale, void* stream) {
    g_last_error[0] = 0;
    if (check_bhn(B, H, N) != BF_OK) return BF_ERR_ARG;
    BfFwdArgs a = base_args(Q, K, V, B, H, N, d, scale, stream);
    a.o = O;
    a.lse = lse;
    a.row_max = row_max;
    return bf_fwd_launch(&a);
}

extern "C" int blackflash_fwd_causal(const void* Q, const void* K, const void* V, void* O, float* lse,
                                     float* row_max, int B, int H, int N, int d, float scale, void* stream) {
    g_last_error[0] = 0;
    if (check_bhn(B, H, N) != BF_OK) return BF_ERR_ARG;
    BfFwdArgs a = base_args(Q, K, V, B, H, N, d, scale, stream);
    a.o = O;
    a.lse = lse;
    a.row_max = row_max;
    a.causal = 1;
    return bf_fwd_launch(&a);
}

extern "C" int blackflash_fwd_partial(const void* Q, const void* K, const void* V, float* O_f32, float* lse,
                                      long long BH, int Nq, int Nkv, int d, float scale, void* stream) {
    g_last_error[0] = 0;
    if (!O_f32 || !lse) return bf_set_error(BF_ERR_ARG, "partial mode needs O_f32 and lse");
    BfFwdArgs a;
    memset(&a, 0, sizeof(a));
    a.q = Q;
    a.k = K;
    a.v = V;
    a.o_f32 = O_f32;
    a.lse = lse;
    a.bh = BH;
    a.n_q = Nq;
    a.n_kv = Nkv;
    a.d = d;
    a.scale = scale;
    a.stream = stream;
    return bf_fwd_launch(&a);
}

extern "C" long long blackflash_bwd_workspace_bytes(int B, int H, int N, int d) {
    if (B <= 0 || H <= 0 || N <= 0 || d != 64) return 0;
    return bf_bwd_workspace_bytes((long long)B * H, N);
}

extern "C" int blackflash_bwd(const void* Q, const void* K, const void* V, const void* O, const void* dO,
                              const float* lse, void* dQ, void* dK, void* dV, void* workspace,
                              long long workspace_bytes, int B, int H, int N, int d, float scale, void* stream) {
    g_last_error[0] = 0;
    if (check_bhn(B, H, N) != BF_OK) return BF_ERR_ARG;
    if (d != 64) return bf_set_error(BF_ERR_ARG, "the backward supports d=64");
    if (workspace_bytes < bf_bwd_workspace_bytes((long long)B * H, N))
        return bf_set_error(BF_ERR_ARG, "workspace smaller than blackflash_bwd_workspace_bytes()");
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
    a.workspace = workspace;
    a.bh = (long long)B * H;
    a.n = N;
    a.d = d;
    a.scale = scale;
    a.stream = stream;
    return bf_bwd_launch(&a);
}

extern "C" int blackflash_fwd_partial_blocks(const void* Q, const void* Kg, const void* Vg, float* O_f32, float* lse,
                                             long long BH, int Nq, int n_blocks, int block_rows, int skip, int d,
                                             float scale, void* stream) {
    g_last_error[0] = 0;
    if (!O_f32 || !lse) return bf_set_error(BF_ERR_ARG, "partial mode needs O_f32 and lse");
    if (block_rows % 128) return bf_set_error(BF_ERR_ARG, "block_rows must be a multiple of 128");
    if (n_blocks < 1 || block_rows <= 0 || skip < -1 || skip >= n_blocks || (skip >= 0 && n_blocks == 1))
        return bf_set_error(BF_ERR_ARG, "need n_blocks >= 1, block_rows >= 1, -1 <= skip < n_blocks, a block left");
    const long long n_kv = (long long)(n_blocks - (skip >= 0)) * block_rows;
    if (n_kv > 0x7fffffffLL) return bf_set_error(BF_ERR_ARG, "too many KV rows");
    BfFwdArgs a;
    memset(&a, 0, sizeof(a));
    a.q = Q;
    a.k = Kg;
    a.v = Vg;
    a.o_f32 = O_f32;
    a.lse = lse;
    a.bh = BH;
    a.n_q = Nq;
    a.n_kv = (int)n_kv;
    a.d = d;
    a.scale = scale;
    a.stream = stream;
    a.kv_blocks = n_blocks;
    a.kv_block_rows = block_rows;
    a.kv_skip = skip;
    return bf_fwd_launch(&a);
}

extern "C" int blackflash_fwd_timeout_probe(const void* Q, const void* K, const void* V, void* O, int B, int H, int N,
                                            int d, float scale, unsigned long long timeout_ns, void* stream) {
    g_last_error[0] = 0;
    if (check_bhn(B, H, N) != BF_OK) return BF_ERR_ARG;
    if (timeout_ns == 0) return bf_set_error(BF_ERR_ARG, "timeout_ns must be > 0");
    BfFwdArgs a = base_args(Q, K, V, B, H, N, d, scale, stream);
    a.o = O;
    a.timeout_ns = timeout_ns;
    a.skip_k_loads = 1;
    return bf_fwd_launch(&a);
}

extern "C" int blackflash_fwd_debug_s(const void* Q, const void* K, const void* V, void* O, float* dbg_s, int B, int H,
                                      int N, int d, float scale, void* stream) {
    g_last_error[0] = 0;
    if (check_bhn(B, H, N) != BF_OK) return BF_ERR_ARG;
    BfFwdArgs a = base_args(Q, K, V, B, H, N, d, scale, stream);
    a.o = O;
    a.dbg_s = dbg_s;
    return bf_fwd_launch(&a);
}

extern "C" int blackflash_fwd_trace(const void* Q, const void* K, const void* V, void* O, long long* trace,
                                    int trace_cta, int B, int H, int N, int d, float scale, void* stream) {
    g_last_error[0] = 0;
    if (check_bhn(B, H, N) != BF_OK) return BF_ERR_ARG;
    if (!trace) return bf_set_error(BF_ERR_ARG, "trace buffer required");
    BfFwdArgs a = base_args(Q, K, V, B, H, N, d, scale, stream);
    a.o = O;
    a.trace = trace;
    a.trace_cta = trace_cta;
    return bf_fwd_launch(&a);
}

// Reference-signature launcher (include/flash_attn.cuh:22-32 of the reference).
void flash_attn_naive_launch(const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V,
                             __nv_bfloat16* O, float* l, float* m, int B, int H, int N, int d, float scale,
                             cudaStream_t stream) {
    const int rc = blackflash_fwd(Q, K, V, O, l, m, B, H, N, d, scale, reinterpret_cast<void*>(stream));
    if (rc != BF_OK) fprintf(stderr, "flash_attn_naive_launch: %s\n", blackflash_last_error());
}
