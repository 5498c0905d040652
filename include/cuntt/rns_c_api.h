/*
 * rns_c_api.h -- RNS (multi-modulus) word64 NTT C ABI of cubutterfly_b200.
 *
 * Drop-in replacement for the reference's include/cuntt/rns_c_api.h:12-36:
 * same opaque handle, entry points, status codes (0 ok, 1 invalid argument or
 * state, 2 runtime failure), thread-local error text and strict schema-v1
 * config JSON ({"schema_version", "log_n", "inverse", "ring", "input_order",
 * "output_order", "domains": [{"modulus", "root"}], "polynomials":
 * [{"domain", "input_offset", "output_offset"}]}, unknown keys rejected, as
 * reference src/rns_tuning.cpp:127-146).  Roots describe the forward
 * transform: a primitive 2N-th root for negacyclic rings, N-th for cyclic.
 * All functions catch C++ exceptions; handles must not be shared between
 * threads concurrently.
 */
#ifndef CUBUTTERFLY_B200_RNS_C_API_H
#define CUBUTTERFLY_B200_RNS_C_API_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CUBUTTERFLY_RNS_API __attribute__((visibility("default")))

typedef struct cubutterflyRnsPlanOpaque* cubutterflyRnsPlan;

/* reference rns_c_api.h:15 */
CUBUTTERFLY_RNS_API const char* cubutterflyRnsLastError(void);
/* reference rns_c_api.h:16.  Validates the request (prime moduli < 2^63,
 * primitive roots of the required order, disjoint output intervals) and
 * uploads per-domain tables. */
CUBUTTERFLY_RNS_API int cubutterflyRnsCreate(const char* config_json, cubutterflyRnsPlan* result);
/* reference rns_c_api.h:20-22.  placement: 0 separate, 1 in-place; policy:
 * 0 prefer, 1 require, 2 refresh a cached mapping in cache_directory (empty
 * disables persistence).  Runs outside stream capture. */
CUBUTTERFLY_RNS_API int cubutterflyRnsPrepare(cubutterflyRnsPlan plan, int placement, const char* cache_directory,
                                              int policy, unsigned repetitions, void* stream);
/* reference rns_c_api.h:27-28.  Asynchronous, allocation-free; canonical
 * residues in, canonical residues out; pointers 8-byte aligned; aliasing must
 * match the prepared placement. */
CUBUTTERFLY_RNS_API int cubutterflyRnsExecute(cubutterflyRnsPlan plan, const uint64_t* input, uint64_t* output,
                                              void* stream);
/* reference rns_c_api.h:31.  Two-call size query (buffer NULL). */
CUBUTTERFLY_RNS_API int cubutterflyRnsInfoJson(cubutterflyRnsPlan plan, char* buffer, size_t* bytes);
/* reference rns_c_api.h:32 */
CUBUTTERFLY_RNS_API int cubutterflyRnsDestroy(cubutterflyRnsPlan plan);

#ifdef __cplusplus
}
#endif

#endif /* CUBUTTERFLY_B200_RNS_C_API_H */
