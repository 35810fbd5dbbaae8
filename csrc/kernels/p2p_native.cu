// Native device Send/Recv over NVLink peer memory (BCCL_P2P_NATIVE=1; NCCL's send/recv is the
// default path).
//
// One launch runs every Send and Recv of a group on this rank. Each directed pair's operations
// are cut into chunks that travel on the pair's channels (p2p_sched.h); a channel is one CTA on
// the sender and one on the receiver, working through a ring of kP2pSlots inbox slots in the
// receiver's P2P region:
//
//   sender CTA:   wait until the receiver consumed the message that last used the slot
//                 (consumed flag in the sender's own control region), store the chunk into the
//                 receiver's slot over NVLink, fence, raise the receiver's posted flag;
//   receiver CTA: wait for the posted flag (own control region), copy the slot into the user
//                 buffer, fence, raise the sender's consumed flag.
//
// Flags and the per-channel message counters in DevState are monotonic across launches, so a
// launch needs no barrier at its start or end and a CUDA graph can replay it. Every wait is
// bounded (wait_flag_geq): on a timeout or an abort the CTA records the error and returns, and
// the host reports it. Every CTA of a launch must be resident at once (a sender CTA may wait for
// a receiver CTA of the peer that waits for data from another pair): at most kP2pMaxRoles
// (112) CTAs of 512 threads, one per SM.
#include "kernels/common.cuh"
#include "kernels/launch.h"
#include "kernels/p2p_sched.h"

namespace bccl {
namespace dev {
namespace {

struct P2pNativeParams {
    DevComm comm;
    int nroles;
    int nops;
    P2pNativeRole roles[kP2pMaxRoles];
    P2pNativeOp ops[kP2pMaxOps];
};

static_assert(sizeof(P2pNativeParams) <= 32764, "kernel parameter limit");

__device__ __forceinline__ uint64_t* p2p_flag(char* uc_base, size_t off, int rank, int ch) {
    return reinterpret_cast<uint64_t*>(uc_base + off) + (size_t)rank * kP2pMaxChannels + ch;
}

constexpr int kPhaseP2pSend = 20;  // error record phase: sender waited for a free slot
constexpr int kPhaseP2pRecv = 21;  // receiver waited for a posted chunk

__global__ void __launch_bounds__(512, 1) p2p_native_kernel(const __grid_constant__ P2pNativeParams p) {
    const DevComm& c = p.comm;
    const P2pNativeRole role = p.roles[blockIdx.x];
    const int me = c.rank, peer = role.peer, ch = role.channel;
    const bool send = role.dir == 0;
    unsigned long long* counter = send ? &c.state->p2p_sent[peer][ch] : &c.state->p2p_recvd[peer][ch];
    const uint64_t base = load_state_u64(counter);
    // The flag this CTA waits on lives in its own control region; the one it raises in the peer's.
    const uint64_t* wait_on = p2p_flag(c.uc[me], send ? kP2pConsumedOff : kP2pPostedOff, peer, ch);
    uint64_t* raise = p2p_flag(c.uc[peer], send ? kP2pPostedOff : kP2pConsumedOff, me, ch);
    // Inbox slots of this channel: in the receiver's P2P region, indexed by the sender's rank.
    char* inbox = (send ? c.uc[peer] : c.uc[me]) + kCtrlBytes + c.data_bytes;
    const int src = send ? me : peer;
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        s_ok = 1;
        trace(c, 0, kTrBegin, (int)(base & 0x7fffffffull));
    }
    __syncthreads();
    uint64_t msg = base;
    P2pCursor cur(role.op_begin, role.nch, ch);
    int i = 0;
    unsigned long long off = 0, len = 0;
    while (s_ok && cur.next(p.ops, role.op_end, &i, &off, &len)) {
        char* slot = inbox + P2pSlotOffset(src, ch, (int)(msg % kP2pSlots));
        if (threadIdx.x == 0) {
            bool ok;
            if (send) {  // message msg - kP2pSlots used this slot: it must have been consumed
                ok = msg < (uint64_t)kP2pSlots ||
                     wait_flag_geq(c, wait_on, msg + 1 - kP2pSlots, peer, kPhaseP2pSend);
            } else {
                ok = wait_flag_geq(c, wait_on, msg + 1, peer, kPhaseP2pRecv);
            }
            if (!ok) s_ok = 0;
        }
        __syncthreads();
        if (!s_ok) break;
        if (send) {
            cta_copy(slot, p.ops[i].buf + off, (size_t)len, false);
        } else {
            cta_copy(p.ops[i].buf + off, slot, (size_t)len, true);  // written by the peer: bypass L1
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            fence_acq_rel_sys();  // the chunk's stores (or the slot's reads) before the flag
            st_relaxed_sys_flag(raise, msg + 1);
        }
        ++msg;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        trace(c, 0, kTrEnd, (int)(msg - base));
        if (s_ok) *counter = msg;
    }
}

}  // namespace
}  // namespace dev

cudaError_t LaunchP2pNative(const DevComm& c, const P2pNativeOp* ops, int nops, const P2pNativeRole* roles,
                            int nroles, cudaStream_t stream) {
    using namespace dev;
    if (nroles <= 0 || nroles > kP2pMaxRoles || nops <= 0 || nops > kP2pMaxOps || c.nranks < 2) {
        return cudaErrorInvalidValue;
    }
    P2pNativeParams p;
    p.comm = c;
    p.nroles = nroles;
    p.nops = nops;
    for (int r = 0; r < nroles; ++r) {
        const P2pNativeRole& q = roles[r];
        if (q.peer < 0 || q.peer >= c.nranks || q.peer == c.rank || q.dir < 0 || q.dir > 1 || q.nch < 1 ||
            q.nch > kP2pMaxChannels || q.channel < 0 || q.channel >= q.nch || q.op_begin < 0 || q.op_end > nops ||
            q.op_begin > q.op_end) {
            return cudaErrorInvalidValue;
        }
        p.roles[r] = q;
    }
    for (int i = 0; i < nops; ++i) p.ops[i] = ops[i];
    p2p_native_kernel<<<nroles, 512, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace bccl
