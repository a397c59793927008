// The exchange step of a KV-range-sharded decode over NVLink peer memory, in place of an NCCL
// all-gather followed by the merge kernel: one small kernel per rank stores its per-head
// (max, sum, o) partials straight into every rank's gather buffer (CUDA IPC mappings: P2P stores
// over NVLink / NVSwitch), raises its flag in each (a system-scope release after a system
// fence), waits until every rank's flag in its own buffer carries this step's sequence number
// (a system-scope acquire, bounded: after about a second it records kErrTimeout), and merges the
// partials of the ranks whose flag carries it, in rank order, with the merge kernel's
// arithmetic. A rank whose flag never came is left out of the merge (its slot holds partials of
// an earlier step): the output is then incomplete and the error word says so. The ranks' step
// counters have diverged by then, so every later step would wait in vain: the host resets every
// rank's header together (fa_peer_reset on each rank between two barriers) before the next.
//
// Buffer of each rank (fa_peer_buffer_bytes): a 256-byte header (the step counter at 0, the
// flags [2][kMaxPeers] at 128), then the partials [2][world][heads][head_dim + 2] f32. Steps
// alternate between the two halves (sequence parity): a rank cannot start step s + 2 before every
// rank has published step s + 1, which each does only after merging step s, so a half is never
// written while it is read. The sequence number lives in device memory (the counter), so a CUDA
// graph that replays the step stays in step with the other ranks.
#include <cuda_runtime.h>

#include "fa_launch.cuh"
#include "fa_peer.h"

namespace fa {

namespace {

__device__ __forceinline__ void store_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned load_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

constexpr int kPeerThreads = 256;

__global__ void __launch_bounds__(kPeerThreads) peer_merge_kernel(const PeerMergeArgs a) {
  __shared__ unsigned s_seq;
  __shared__ unsigned s_missing;  // ranks whose flag did not arrive in time (bit per rank)
  const int pitch = a.heads * (a.head_dim + 2);  // floats of one rank's partials
  unsigned char* mine = a.bufs[a.rank];
  if (threadIdx.x == 0) {
    unsigned* counter = reinterpret_cast<unsigned*>(mine);
    s_seq = *counter + 1;  // this rank's kernels of this exchange run one at a time (one stream)
    *counter = s_seq;
    s_missing = 0u;
  }
  __syncthreads();
  const unsigned seq = s_seq;
  const int half = int(seq & 1u);
  // 1. this rank's partials into slot `rank` of every rank's buffer (its own included)
  for (int p = 0; p < a.world; ++p) {
    float* dst = reinterpret_cast<float*>(a.bufs[p] + kPeerHeaderBytes) +
                 (int64_t(half) * a.world + a.rank) * pitch;
    for (int e = threadIdx.x; e < pitch; e += kPeerThreads) dst[e] = a.partials[e];
  }
  __threadfence_system();  // the partials are visible to every GPU before any flag is
  __syncthreads();
  // 2. this rank's flag in every buffer
  if (threadIdx.x < a.world) {
    unsigned* flags = reinterpret_cast<unsigned*>(a.bufs[threadIdx.x] + kPeerFlagsOffset);
    store_release_sys(flags + half * kMaxPeers + a.rank, seq);
  }
  // 3. every rank's flag in this rank's buffer (bounded wait)
  if (threadIdx.x < a.world) {
    const unsigned* flag =
        reinterpret_cast<const unsigned*>(mine + kPeerFlagsOffset) + half * kMaxPeers + threadIdx.x;
    if (load_acquire_sys(flag) != seq) {
      const long long start = clock64();
      while (load_acquire_sys(flag) != seq) {
        if (clock64() - start > kWaitCycles) {
          atomicOr(a.err, kErrTimeout);
          atomicOr(&s_missing, 1u << threadIdx.x);
          break;
        }
      }
    }
  }
  __syncthreads();
  __threadfence_system();
  // 4. the merge, ranks in order (merge_partials_kernel's arithmetic); the partials are read
  // through L2 (written by other GPUs since this SM may have cached the half two steps ago)
  const float* data = reinterpret_cast<const float*>(mine + kPeerHeaderBytes) +
                      int64_t(half) * a.world * pitch;
  const int d = a.head_dim;
  const unsigned missing = s_missing;
  for (int idx = threadIdx.x; idx < a.heads * d; idx += kPeerThreads) {
    const int h = idx / d, e = idx % d;
    float mm = -INFINITY;
    for (int s = 0; s < a.world; ++s)
      if (!(missing >> s & 1u)) mm = fmaxf(mm, __ldcg(data + int64_t(s) * pitch + h * (d + 2)));
    float ll = 0.0f, oo = 0.0f;
    for (int s = 0; s < a.world; ++s) {
      if (missing >> s & 1u) continue;
      const float* p = data + int64_t(s) * pitch + h * (d + 2);
      const float m = __ldcg(p);
      const float f = m == -INFINITY ? 0.0f : exp2f(m - mm);
      ll = fmaf(__ldcg(p + 1), f, ll);
      oo = fmaf(__ldcg(p + 2 + e), f, oo);
    }
    a.out[int64_t(h) * d + e] = ll > 0.0f ? oo / ll : 0.0f;
  }
}

}  // namespace

size_t peer_buffer_bytes(int world, int heads, int head_dim) {
  return size_t(kPeerHeaderBytes) + size_t(2) * world * heads * (head_dim + 2) * sizeof(float);
}

cudaError_t launch_peer_merge(const PeerMergeArgs& args, cudaStream_t stream) {
  peer_merge_kernel<<<1, kPeerThreads, 0, stream>>>(args);
  return cudaGetLastError();
}

}  // namespace fa
