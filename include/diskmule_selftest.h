/*
 * diskmule_selftest.h -- self-tests of the library's failure handling. No counterpart in
 * the reference (its failure tests are host-side: cancellation flags and rollback).
 *
 * dm_selftest_device_wait runs the bounded mbarrier wait that every tensor-core kernel
 * uses on a barrier that nothing arrives on, with a limit of `cycles` SM clocks: the
 * wait gives up, the kernel records a timeout status and returns, and the call returns
 * DM_ERR_TIMEOUT with the context still usable -- the path a stuck copy or MMA would
 * take, exercised without a stuck copy or MMA.
 */
#ifndef DISKMULE_SELFTEST_H
#define DISKMULE_SELFTEST_H

#include <stdint.h>

#include "diskmule_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

DM_API int32_t dm_selftest_device_wait(dm_cuda_context *ctx, int64_t cycles);

#ifdef __cplusplus
}
#endif
#endif
