/*
 * spb_debug.h -- test hooks of libspbatch_b200_debug.so.
 *
 * The debug library is the product library compiled with SPB_DEBUG_HOOKS; it
 * adds this one entry point, which the failure-path tests use to make a
 * bounded device wait run out on purpose.  The product library
 * (libspbatch_b200.so) does not export it, so no setting here can reach a
 * timed or production run.  No counterpart in the reference, whose kernels
 * have no bounded waits (cuda/kernel.cuh:17-41 exits the process on error).
 */
#ifndef SPB_DEBUG_H_
#define SPB_DEBUG_H_

#include "spb.h"

#ifdef __cplusplus
extern "C" {
#endif

enum {
    SPB_DEBUG_TIMEOUT_NS = 1, /* limit of the tensor path's bounded waits, ns (0: the default 2 s) */
    SPB_DEBUG_INJECT = 2,     /* 1: the tensor path's rank-1 CTAs never signal their gate/up results,
                                 so the partner's wait runs out and records error code 4 */
    SPB_DEBUG_TC_NKB = 3,     /* tensor path: K blocks per gate/up stage (1, 2, 4; 0 automatic) */
    SPB_DEBUG_TC_STAGES = 4,  /* tensor path: cap on the ring depth (0 automatic) */
    SPB_DEBUG_TC_HINT_ACC = 5, /* tensor path: suspend hint of the epilogue's accumulator waits, ns */
    SPB_DEBUG_TC_HINT = 6,    /* tensor path: suspend hint of the ring waits, ns */
    SPB_DEBUG_TC_SPLIT_STAGES = 7, /* tensor path: 1 = one ring unit per stage (no half-stage units) */
    SPB_DEBUG_TC_LAUNCH_FLAGS = 8, /* tensor path, launch-overhead measurement: 1 = launch without the
                                      cooperative attribute, 2 = without programmatic dependent launch */
    SPB_DEBUG_TC_DENSE_PERMILLE = 9, /* tensor path: union share of f (per mille) from which whole row
                                        ranges stream (0: the default; above 1000: never) */
};

/* Sets one process-wide hook; applies to launches made after the call. */
int spb_debug_config(int key, long long value);

#ifdef __cplusplus
}
#endif

#endif /* SPB_DEBUG_H_ */
