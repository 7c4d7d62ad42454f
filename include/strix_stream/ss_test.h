/* Test-only hooks of the device-gated mode (same names as the reference library's ss_test.h). Not part of the stable
 * ABI. Each refuses with SS_E_INVALID unless the context was opened with ss_options.dg_test_hooks = 1. */
#ifndef STRIX_STREAM_SS_TEST_H
#define STRIX_STREAM_SS_TEST_H

#include "strix_stream/ss.h"

#ifdef __cplusplus
extern "C" {
#endif

/* A cache-core fault to inject; the tests must catch it (0 = none). Supported here: 1 = an entry published before its
 * copy, 2 = no cover wait of a prefetched unit. Others return SS_E_UNSUPPORTED. */
SS_API ss_status ss_test_dg_mutate(ss_ctx* c, int mutation);
/* Demand misses take at most free_per_token free slots per token; each boundary also evicts the evict_recent most
 * recently used units. 0, 0 = off. */
SS_API ss_status ss_test_dg_pressure(ss_ctx* c, uint32_t free_per_token, uint32_t evict_recent);
/* Checks every ownership invariant of the cache (SS_E_BACKEND naming the first broken rule). */
SS_API ss_status ss_test_dg_check(ss_ctx* c);
/* The library's demand (0) or prefetch (1) stream waits for `event` (a cudaEvent_t). */
SS_API ss_status ss_test_dg_gate(ss_ctx* c, int stream, void* event);
/* Kernel mutations, set before capture: 1 = the wait kernel returns at once, 2 = ss_end skips the completion edge. */
SS_API ss_status ss_test_dg_flags(ss_ctx* c, uint32_t flags);
/* Between tokens: units whose copy is enqueued and not admitted yet. */
SS_API ss_status ss_test_dg_coming(ss_ctx* c, uint32_t* out);
/* Stops the service thread (its next token fails closed). */
SS_API ss_status ss_test_dg_stop_service(ss_ctx* c);

#ifdef __cplusplus
}
#endif

#endif
