/*
 * cubutterfly_b200.h -- extensions of the B200 build beyond the reference ABI.
 *
 * Nothing here replaces a reference entry point; callers of the reference
 * header need none of it.  Symbols use the cubutterflyB200 prefix.
 */
#ifndef CUBUTTERFLY_B200_EXT_H
#define CUBUTTERFLY_B200_EXT_H

#include <cubutterfly/cubutterfly.h>

#ifdef __cplusplus
extern "C" {
#endif

/* CPU-only planner preview (no counterpart in the reference ABI; the
 * reference exposes its static ranking only through a Python subprocess,
 * scripts/rank_static_candidates.py).  Writes a JSON array of every legal
 * mapping of the descriptor, best first, as the DEFAULT policy would rank it
 * under `hardware_json` (a cubutterfly-b200-hardware-v1 object; NULL selects
 * the current device or the builtin B200 profile).  Two-call size protocol. */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200RankMappings(cubutterflyDescriptor_t descriptor,
                                                              const char* hardware_json, char* json,
                                                              size_t* bytes);

/* Device-side status of a plan (no counterpart in the reference ABI): the
 * persistent kernels wait on shared-memory barriers with bounded polls and,
 * instead of trapping, record a nonzero code (1 = a bulk-copy wait expired)
 * in a per-plan device word.  Reads the word after synchronising the
 * handle's stream; `reset` nonzero clears it. */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyB200PlanGetDeviceStatus(cubutterflyHandle_t handle,
                                                                     cubutterflyPlan_t plan, unsigned* status,
                                                                     int reset);

#ifdef __cplusplus
}
#endif

#endif /* CUBUTTERFLY_B200_EXT_H */
