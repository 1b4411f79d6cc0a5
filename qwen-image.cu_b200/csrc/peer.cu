// peer.cu -- the flag barrier of the head-parallel exchanges over peer memory.
//
// qkv_post and the attention epilogue store straight into other ranks'
// buffers (CUDA IPC mappings over NVLink).  Between such a store phase and the
// kernels that read the data, every rank runs this barrier: one thread per
// peer publishes the epoch to that peer's flag word for this rank (release,
// system scope) and then waits for the peer's flag in this rank's own words
// (acquire), giving up after a time limit with an error word instead of
// spinning forever.
#include "qi_internal.h"
#include "sm100.cuh"

namespace qi {
namespace {
__global__ void peer_barrier_kernel(PeerSet ps, int slot, unsigned epoch, int* err) {
  const int q = threadIdx.x;
  if (q >= ps.P) return;
  __threadfence_system();  // this stream's earlier stores before the flag
  unsigned* remote = ps.flags[q] + slot * kMaxRanks + ps.rank;
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(remote), "r"(epoch) : "memory");
  const unsigned* mine = ps.flags[ps.rank] + slot * kMaxRanks + q;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
    if (static_cast<int>(v - epoch) >= 0) break;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      atomicCAS(err, 0, kErrTimeoutPeer);
      break;
    }
    __nanosleep(64);
  }
}
}  // namespace

int peer_barrier_launch(const PeerSet& ps, int slot, unsigned epoch, int* err, cudaStream_t stream) {
  if (ps.P < 2 || ps.P > kMaxRanks || slot < 0 || slot > 1) return QI_ERR_ARG;
  peer_barrier_kernel<<<1, 32, 0, stream>>>(ps, slot, epoch, err);
  return cudaGetLastError() == cudaSuccess ? QI_OK : QI_ERR_CUDA;
}
}  // namespace qi
