/* Allocation-free single-GPU entry point.
 *
 * This entry point has no counterpart in the reference library; it exists for callers of
 * this library that cannot allocate device memory themselves or let a library do it:
 *   - frameworks whose caching allocator owns every byte of device memory and forbid side
 *     allocations (an extra cudaMalloc fragments the pool or fails when it is full);
 *   - latency-critical threads that must not enter the driver's allocation path, since
 *     cudaMalloc/cudaFree may synchronise the device and block for milliseconds;
 *   - tools loaded into a process that must not change its device memory footprint.
 *
 * bcclLocalAllReduceNoAlloc runs the one-rank AllReduce of a batch of tensors (what a
 * communicator with world size 1 computes for each: dst = src, divided by 1 for AVG and
 * multiplied by `scale`) as ONE launch of the push-engine kernel, like a one-rank
 * communicator would, but every piece of scratch memory that kernel needs -- its sequence
 * counters, its error record and its work list -- lives in a fixed file-scope device array
 * of BCCL_NOALLOC_SCRATCH_BYTES bytes instead of memory from cudaMalloc. The caller passes
 * the inputs and the outputs (device pointers). Nothing is allocated: no cudaMalloc,
 * cudaFree or allocating library call, on any call.
 *
 * Limits and rules:
 *   - at most BCCL_NOALLOC_MAX_ITEMS tensors per call (larger batches are rejected with an
 *     error; split them across calls);
 *   - the array exists once per device and every GPU that loads the library holds it until
 *     the process exits;
 *   - the first call on a device looks up the array's device address for that device (with
 *     the device current) and caches it; make that first call before any stream capture
 *     begins on the device. After a cudaDeviceReset the next call looks the address up again;
 *   - all calls on a device share the one array, which keeps the previous call's contents
 *     (the call clears what must start at zero): calls that overlap on the GPU -- on
 *     different streams without ordering between them -- race on the array and must not be
 *     issued.
 * The call is asynchronous on `stream` (0 = legacy default stream) and returns 0 on success,
 * non-zero on an argument or launch error (bcclGetLastError() says which).
 */
#ifndef BCCL_NOALLOC_H_
#define BCCL_NOALLOC_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BCCL_NOALLOC_MAX_ITEMS 1024
#define BCCL_NOALLOC_SCRATCH_BYTES (64 * 1024)

int bcclLocalAllReduceNoAlloc(const void* const* srcs, void* const* dsts, const size_t* counts, int n, int dtype,
                              int op, float scale, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BCCL_NOALLOC_H_ */
