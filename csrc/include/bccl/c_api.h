/* C interface of the library (used by the Python bindings through ctypes, and by any
 * caller that cannot link C++). Every function returns 0 on success and a non-zero code on
 * failure; bcclGetLastError() describes the most recent failure on the calling thread.
 * Buffers are host pointers for host communicators and device pointers for device ones.
 * `stream` arguments apply to device communicators: with has_stream != 0 the call enqueues on
 * that cudaStream_t and returns; with has_stream == 0 it runs on the internal stream and
 * blocks until the result is ready. */
#ifndef BCCL_C_API_H_
#define BCCL_C_API_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct bcclComm* bcclComm_t;

typedef struct {
    int rank;
    int world_size;
    char ip_addr[64];
    uint16_t port;
    int n_channels;
    int device;                 /* -1 = host-memory communicator */
    size_t buffer_bytes;        /* 0 = default */
    int timeout_ms;             /* 0 = default */
    int enable_nvls;
    int enable_nccl_p2p;
    int logical_machine_size;   /* > 0: ranks r and s share a machine iff r/size == s/size */
} bcclConfig;

enum { bcclFloat32 = 0, bcclFloat64 = 1, bcclInt32 = 2, bcclInt64 = 3, bcclBfloat16 = 4, bcclFloat16 = 5 };
enum { bcclSum = 0, bcclMax = 1, bcclMin = 2, bcclAvg = 3 };

int bcclCommCreate(bcclComm_t* comm);
int bcclGetUniqueId(bcclComm_t comm, char ip_addr[64], uint16_t* port);
int bcclCommInit(bcclComm_t comm, const bcclConfig* cfg);
int bcclCommFinalize(bcclComm_t comm);
int bcclCommDestroy(bcclComm_t comm);
/* Collective (MPI_Comm_split): ranks with the same color >= 0 get a new communicator in *out,
 * ranked by (key, rank); a negative color gets *out = NULL. */
int bcclCommSplit(bcclComm_t comm, int color, int key, bcclComm_t* out);
const char* bcclGetLastError(void);
const char* bcclVersion(void);

int bcclCommInfo(bcclComm_t comm, int* rank, int* world, int* local_rank, int* local_size, int* machine_index,
                 int* machine_count, int* n_channels);
int bcclCommLocalRanks(bcclComm_t comm, int* out, int max);
int bcclCommMachineLeaders(bcclComm_t comm, int* out, int max);
int bcclCommNvlsEnabled(bcclComm_t comm);
const char* bcclCommLastAlgorithm(bcclComm_t comm);
unsigned long long bcclCommKernelLaunches(bcclComm_t comm);
const char* bcclCommP2pTransport(bcclComm_t comm, int peer);
const char* bcclCommHostExecutor(bcclComm_t comm);
/* Host communicators: single-copy Send/Recv between ranks of a machine (*enabled) and the number
 * of such messages this rank has received. */
unsigned long long bcclCommHostZeroCopyTransfers(bcclComm_t comm, int* enabled);

int bcclGroupStart(bcclComm_t comm);
int bcclGroupEnd(bcclComm_t comm, uintptr_t stream, int has_stream);

/* algo: 0 auto, 1 one-shot, 2 two-shot, 3 NVLS, 4 ring. */
int bcclAllReduce(bcclComm_t comm, const void* send, void* recv, size_t count, int dtype, int op, float scale, int algo,
                  uintptr_t stream, int has_stream);
/* n AllReduces (same dtype, op and scale) in one call: with grouped != 0 they form one group
 * (GroupStart, n submissions, GroupEnd), so small ones run as a single batched kernel; with
 * grouped == 0 each runs as its own operation, in order. Saves a call per tensor for callers
 * that sync many tensors, e.g. gradient buckets. */
int bcclAllReduceMany(bcclComm_t comm, int n, const void* const* send, void* const* recv, const size_t* counts,
                      int dtype, int op, float scale, int grouped, uintptr_t stream, int has_stream);
int bcclBroadcast(bcclComm_t comm, const void* send, void* recv, size_t count, int dtype, int root, int algo,
                  uintptr_t stream, int has_stream);
int bcclReduce(bcclComm_t comm, const void* send, void* recv, size_t count, int dtype, int op, int root, int algo,
               uintptr_t stream, int has_stream);
int bcclAllGather(bcclComm_t comm, const void* send, void* recv, size_t count, int dtype, uintptr_t stream,
                  int has_stream);
int bcclReduceScatter(bcclComm_t comm, const void* send, void* recv, size_t count, int dtype, int op,
                      uintptr_t stream, int has_stream);
/* The same with an algorithm override (0 auto, 1 one-shot push, 3 NVLS; others mean auto). */
int bcclAllGatherAlgo(bcclComm_t comm, const void* send, void* recv, size_t count, int dtype, int algo,
                      uintptr_t stream, int has_stream);
int bcclReduceScatterAlgo(bcclComm_t comm, const void* send, void* recv, size_t count, int dtype, int op, int algo,
                          uintptr_t stream, int has_stream);
int bcclSend(bcclComm_t comm, const void* buf, size_t count, int dtype, int peer, uintptr_t stream, int has_stream);
int bcclRecv(bcclComm_t comm, void* buf, size_t count, int dtype, int peer, uintptr_t stream, int has_stream);
int bcclSynchronize(bcclComm_t comm);
/* Without synchronising (like ncclCommGetAsyncError): *code = 0, or the failure a device kernel
 * recorded so far (1 timeout, 2 aborted, 3 bad arguments; 1 after a failed host operation). */
int bcclCommGetAsyncError(bcclComm_t comm, int* code);
int bcclBarrier(bcclComm_t comm);
/* Aborts the communicator's operations in flight; callable from any thread (like ncclCommAbort).
 * Host waits return at once, device waits within about a millisecond; afterwards only
 * bcclCommFinalize / bcclCommDestroy are meaningful. */
int bcclCommAbort(bcclComm_t comm);
void* bcclSymmetricAlloc(bcclComm_t comm, size_t bytes);
int bcclSymmetricFree(bcclComm_t comm, void* ptr);
/* Collective registration of existing device memory for zero-copy collectives (like
 * ncclCommRegister); every rank passes its own buffer of the same size. */
int bcclCommRegister(bcclComm_t comm, void* ptr, size_t bytes);
int bcclCommDeregister(bcclComm_t comm, void* ptr);

/* Failure-detection self-test: runs a kernel whose bounded wait can never be satisfied and
 * returns the error code it recorded (1 = timeout) or -1 if it could not run. */
int bcclDebugWaitProbe(bcclComm_t comm, int timeout_ms);

/* Transport probe: copy bandwidth in GB/s for mode 0 local, 1 write to peer, 2 read from peer,
 * 3 multimem.st (peers must be idle). */
double bcclDebugBandwidth(bcclComm_t comm, int mode, int peer, size_t bytes, int ctas, int iters);

/* The device-side sequence counters after the work queued so far (synchronises the device):
 * out[0..6) = round, barrier, NVLS round, ring message, fused-TP launch counters and the
 * finished-CTA count of the current launch (0 between launches). Every rank must hold the same
 * values after the same calls; tests compare them across ranks. */
int bcclDebugDeviceState(bcclComm_t comm, unsigned long long* out);

/* Device trace (enabled with BCCL_TRACE=<records>): writes a Chrome trace JSON and resets the
 * buffer; returns the number of records or -1 when tracing is off. */
long bcclTraceDump(bcclComm_t comm, const char* path);

/* Tensor-core GEMM (sm_100a tcgen05): C[M,N] = act(A[M,K] * B[N,K]^T), bf16 in/out, f32
 * accumulation; act 0 = none, 1 = SiLU. Asynchronous on `stream`. bcclGemmCheckError()
 * synchronises the current device and returns (and clears) the kernels' error word. */
int bcclGemmBf16(const void* A, const void* B, void* C, int M, int N, int K, int ldc, int act, void* stream);
int bcclGemmCheckError(void);
/* 1 when the GEMMs use 2-SM (cta_group::2) 256x256 tiles, 0 for 1-SM 128x256 tiles. */
int bcclGemmUsesPair(void);
/* Columns of C per tile for an m x n GEMM (256, or 224 with BCCL_GEMM_BN=224|auto on 2-SM tiles). */
int bcclGemmTileWidth(int m, int n);

/* Fused tensor-parallel GEMMs on a device communicator (bf16, one kernel each):
 *   bcclTpAllGatherGemm: y[nranks*ms, n] = act(AllGather(x[ms, k]) * w[n, k]^T)
 *   bcclTpGemmReduceScatter: out[ms, n] = this rank's rows of sum over ranks of h[nranks*ms, k] * w[n, k]^T
 * ms must be a multiple of 128 (at most 64*128), k and n multiples of 8. Every rank calls them together. */
int bcclTpAllGatherGemm(bcclComm_t comm, const void* x, const void* w, void* y, int ms, int k, int n, int act,
                        uintptr_t stream, int has_stream);
int bcclTpGemmReduceScatter(bcclComm_t comm, const void* h, const void* w, void* out, int ms, int k, int n,
                            uintptr_t stream, int has_stream);

/* Planner white-box hooks (used by tests): sorts `n` tasks described by parallel arrays and
 * writes the resulting permutation (indices into the input) to `order`. */
int bcclPlannerSort(int rank, int world, int n, const int* func, const size_t* count, const int* dtype, const int* op,
                    const int* root, const int* peer, int* order);
int bcclPlannerP2pRound(int func, int rank, int peer, int world);
/* Native device Send/Recv schedule hooks (used by tests). bcclP2pChannels: channels of a
 * directed pair moving `pair_bytes` in one group. bcclP2pPlan: the chunks channel `ch` of `nch`
 * carries for operations of sizes bytes[0..nops), in message order: operation index, byte offset
 * and length of each (at most max_out); returns how many, or -1 on bad arguments. */
int bcclP2pChannels(unsigned long long pair_bytes);
/* Low-latency kernel hook (used by tests): the line epoch of the launch that follows `seq`
 * earlier low-latency launches of a communicator. */
unsigned int bcclLLEpoch(unsigned long long seq);
int bcclP2pPlan(const unsigned long long* bytes, int nops, int nch, int ch, int max_out, int* op_out,
                unsigned long long* off_out, unsigned long long* len_out);
int bcclPlannerValidate(int rank, int world, int func, size_t count, int dtype, int op, int root, int peer,
                        int has_send, int has_recv);
int bcclPlannerChoose(int func, int dtype, int op, size_t bytes, int world, int nvls_ok, int max_ctas, int* algo,
                      int* ctas);

#ifdef __cplusplus
}
#endif

#endif /* BCCL_C_API_H_ */
