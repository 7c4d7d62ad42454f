/* CPU restatement of the reference's hot-path arithmetic (TEST INFRASTRUCTURE ONLY: the tests, smoke() and bench.py's
 * cpu_baseline leg call it as the checker; the product library never links it). Each function names the reference
 * file:line it restates. Pinned against the reference's own known answers (tests/test_core.cpp:64-82) and against
 * the reference's compiled sources (oracle/_ref/libtsref.so) by tests/test_oracle.py. */
#ifndef TSB_ORACLE_H
#define TSB_ORACLE_H
#include <stddef.h>
#include <stdint.h>

/* XXH64 of len bytes (xxh64.cpp:39-112): 4 lanes over 32-byte stripes, little-endian reads, tail 8 / 4 / 1. */
uint64_t orc_xxh64(const void* data, size_t len, uint64_t seed);
/* XXH64 of the concatenation of n spans (a unit's parts back to back). */
uint64_t orc_xxh64_spans(const void* const* ptrs, const uint64_t* lens, uint32_t n, uint64_t seed);
/* The synthetic byte stream of the reference fixtures (tests/fixture.hpp:16-22): byte i of file `file_id`. */
void orc_fill_bytes(uint64_t file_id, uint64_t first, uint64_t n, uint8_t* out);
/* The GPU tests' byte check (tests/test_dg_cuda.cu:103-114): sum over i of byte[i] * (i % 251 + 1). */
uint64_t orc_checksum(const uint8_t* p, uint64_t n);
/* The export kernel's record (dg_kernels.cu:49-87): the miss mask of n ids against a slot table (bit i set when id i
 * is in range and slot_of[base + id] < 0); *bad = 1 when an id is out of range. */
uint64_t orc_export_mask(const int32_t* slot_of, uint32_t base, uint32_t units, const int32_t* ids, uint32_t n,
                         uint32_t* bad);
/* ss_dg_slot (ss.h:952-962): the slot engine kernels read, the guard on abort, range or absence. */
int32_t orc_dg_slot(const int32_t* slot_of, const uint32_t* unit_base, uint32_t g, int32_t id, uint32_t guard,
                    uint32_t abort_flag, uint32_t* absent_err);
#endif
