// Internal launch descriptor shared by the C-ABI wrappers and the kernel file.
#pragma once
#include <stdint.h>

#include "../../include/blackflash_b200_diag.h"

struct BfFwdArgs {
    const void* q;
    const void* k;
    const void* v;
    void* o;          // bf16 [BH, n_q, 64] or null when o_f32 is set
    float* o_f32;     // fp32 [BH, n_q, 64] partial-mode output, or null
    float* lse;       // [BH, n_q] or null
    float* row_max;   // [BH, n_q] or null
    long long bh;
    int n_q;
    int n_kv;
    int d;
    float scale;
    void* stream;
    unsigned long long timeout_ns;  // 0 = default
    float* dbg_s;
    int skip_k_loads;
    long long* trace;
    int trace_cta;
    int causal;  // 1: key j visible to query i only if j <= i
    // Blocked KV (sequence-parallel gather): K and V are [kv_blocks, bh, kv_block_rows, 64]
    // and the slice's keys are the concatenation of every block except kv_skip (-1: none).
    // kv_blocks == 0 means the plain [bh, n_kv, 64] layout.
    int kv_blocks;
    int kv_block_rows;
    int kv_skip;
};

int bf_fwd_launch(const BfFwdArgs* a);

struct BfBwdArgs {
    const void* q;
    const void* k;
    const void* v;
    const void* o;
    const void* dout;
    const float* lse;  // [BH, N] natural-log logsumexp of the forward
    void* dq;
    void* dk;
    void* dv;
    void* workspace;   // bf_bwd_workspace_bytes(bh, n) bytes, 16-byte aligned
    long long bh;
    int n;
    int d;
    float scale;
    void* stream;
    unsigned long long timeout_ns;  // 0 = default
};

long long bf_bwd_workspace_bytes(long long bh, int n);
int bf_bwd_launch(const BfBwdArgs* a);
int bf_set_error(int code, const char* msg);
