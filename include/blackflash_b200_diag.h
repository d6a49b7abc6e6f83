/*
 * BlackFlash-B200 test and diagnostic hooks. They are exported by the same
 * library as the C ABI in blackflash_b200.h but are not part of it: they exist
 * for the parity and failure-detection tests and for pipeline tracing, and may
 * change without an ABI version bump. None has a counterpart in the reference.
 * Return codes and blackflash_last_error() as in blackflash_b200.h.
 */
#ifndef BLACKFLASH_B200_DIAG_H
#define BLACKFLASH_B200_DIAG_H

#include "blackflash_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/*
 * Test hook: the same launch as blackflash_fwd, except that the producer never
 * issues the K loads. The consumers' bounded waits therefore run out after
 * timeout_ns, the kernel returns early, and blackflash_status reports the
 * site. No fault or hang is involved. O is left undefined.
 */
int blackflash_fwd_timeout_probe(const void* Q, const void* K, const void* V, void* O, int B, int H, int N, int d,
                                 float scale, unsigned long long timeout_ns, void* stream);

/* Test hook: raw fp32 S = Q K^T of the first 128x128 tile (CTA 0), written to dbg_s. */
int blackflash_fwd_debug_s(const void* Q, const void* K, const void* V, void* O, float* dbg_s, int B, int H, int N,
                           int d, float scale, void* stream);

/*
 * Diagnostic hook: the same launch as blackflash_fwd, built with pipeline event
 * stamps. For CTA `trace_cta` it writes clock64() offsets into trace[0, 4 * 512)
 * (int64, caller-zeroed): trace[role * 512 + step * 8 + event] for the CTA's
 * first 64 KV steps, roles 0/1 = softmax warpgroups, 2 = MMA issuer, 3 = TMA
 * producer. For every CTA c it also writes the global timer (ns) at entry, after
 * set-up, when its first S tile is ready and at exit into trace[4 * 512 + 4 c + k],
 * so the buffer holds 4 * 512 + 4 * (number of SMs) entries.
 */
int blackflash_fwd_trace(const void* Q, const void* K, const void* V, void* O, long long* trace, int trace_cta, int B,
                         int H, int N, int d, float scale, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BLACKFLASH_B200_DIAG_H */
