// The exchange step of a KV-range-sharded decode over NVLink peer memory, in place of an NCCL
// all-gather followed by the merge kernel: one small kernel per rank, a CTA per query head,
// stores the head's (max, sum, o) partials straight into every rank's gather buffer (CUDA IPC
// mappings: P2P stores over NVLink / NVSwitch), then waits until every rank's partials of the
// head have landed in its own buffer and merges them in rank order with the merge kernel's
// arithmetic. The heads are independent: each CTA keeps its own step counter.
//
// Each value travels as one 64-bit word, the step's sequence number in its high half and the
// f32 bits in its low half. A naturally aligned 64-bit store lands whole, so a reader knows a
// value has arrived by its own word: no flag, and no system-scope fence between the data and a
// flag (two NVLink round trips fewer per step). The wait is bounded: a rank whose words have not
// all arrived after about a second is recorded in the error word (kErrTimeout) and left out of
// the merge (its slot holds words of an earlier step), so the output is incomplete and the host
// learns it from fa_device_status. The ranks' step counters have diverged by then: the host
// clears every rank's buffer together (fa_peer_reset between two barriers) before the next step.
//
// Buffer of each rank (fa_peer_buffer_bytes): a 256-byte header (the step counter of head h at
// word h, so at most 64 heads), then the words [2][world][heads][head_dim + 2]. Steps alternate
// between the two halves (sequence parity): a head's CTA cannot start step s + 2 before every
// rank has published the head's step s + 1, which each does only after it has read step s, so a
// half is never written while it is read. The sequence numbers live in device memory (the
// counters), so a CUDA graph that replays the step stays in step with the other ranks.
#include <cuda_runtime.h>

#include "fa_launch.cuh"
#include "fa_peer.h"

namespace fa {

namespace {

__device__ __forceinline__ unsigned long long load_relaxed_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

constexpr int kPeerThreads = 128;

__global__ void __launch_bounds__(kPeerThreads) peer_merge_kernel(const PeerMergeArgs a) {
  __shared__ unsigned s_seq;
  __shared__ unsigned s_missing;  // ranks whose words did not all arrive in time (bit per rank)
  const int h = blockIdx.x;                      // this CTA's query head
  const int d = a.head_dim;
  const int pitch = a.heads * (d + 2);           // words of one rank's partials
  const int row = h * (d + 2);                   // the head's words within them
  unsigned char* mine = a.bufs[a.rank];
  if (threadIdx.x == 0) {
    unsigned* counter = reinterpret_cast<unsigned*>(mine) + h;
    s_seq = *counter + 1;  // this rank's kernels of this exchange run one at a time (one stream)
    *counter = s_seq;
    s_missing = 0u;
  }
  __syncthreads();
  const unsigned seq = s_seq;
  const int half = int(seq & 1u);
  const unsigned long long stamp = static_cast<unsigned long long>(seq) << 32;
  // 1. this rank's partials of the head, stamped, into slot `rank` of every rank's buffer (its
  // own included), each rank's destinations in a different order so that the links share the load
  for (int i = 0; i < a.world; ++i) {
    const int p = (a.rank + i) % a.world;
    unsigned long long* dst = reinterpret_cast<unsigned long long*>(a.bufs[p] + kPeerHeaderBytes) +
                              (int64_t(half) * a.world + a.rank) * pitch + row;
    for (int e = threadIdx.x; e < d + 2; e += kPeerThreads)
      dst[e] = stamp | __float_as_uint(a.partials[row + e]);
  }
  // 2. every rank's words of the head for this step in this rank's buffer (bounded wait)
  const unsigned long long* words =
      reinterpret_cast<const unsigned long long*>(mine + kPeerHeaderBytes) +
      int64_t(half) * a.world * pitch + row;
  for (int s = 0; s < a.world; ++s) {
    const unsigned long long* slot = words + int64_t(s) * pitch;
    for (int e = threadIdx.x; e < d + 2; e += kPeerThreads) {
      if (unsigned(load_relaxed_sys(slot + e) >> 32) == seq) continue;
      const long long start = clock64();
      bool late = false;
      while (unsigned(load_relaxed_sys(slot + e) >> 32) != seq) {
        if (clock64() - start > kWaitCycles) {
          late = true;
          break;
        }
      }
      if (late) {
        atomicOr(a.err, kErrTimeout);
        atomicOr(&s_missing, 1u << s);
        break;  // this rank is left out: its other words need no wait
      }
    }
  }
  __syncthreads();
  // 3. the merge, ranks in order (merge_partials_kernel's arithmetic), of the ranks whose every
  // word of the head arrived
  const unsigned missing = s_missing;
  auto value = [&](int s, int i) {
    return __uint_as_float(unsigned(load_relaxed_sys(words + int64_t(s) * pitch + i)));
  };
  for (int e = threadIdx.x; e < d; e += kPeerThreads) {
    float mm = -INFINITY;
    for (int s = 0; s < a.world; ++s)
      if (!(missing >> s & 1u)) mm = fmaxf(mm, value(s, 0));
    float ll = 0.0f, oo = 0.0f;
    for (int s = 0; s < a.world; ++s) {
      if (missing >> s & 1u) continue;
      const float m = value(s, 0);
      const float f = m == -INFINITY ? 0.0f : exp2f(m - mm);
      ll = fmaf(value(s, 1), f, ll);
      oo = fmaf(value(s, 2 + e), f, oo);
    }
    a.out[int64_t(h) * d + e] = ll > 0.0f ? oo / ll : 0.0f;
  }
}

}  // namespace

size_t peer_buffer_bytes(int world, int heads, int head_dim) {
  return size_t(kPeerHeaderBytes) +
         size_t(2) * world * heads * (head_dim + 2) * sizeof(unsigned long long);
}

cudaError_t launch_peer_merge(const PeerMergeArgs& args, cudaStream_t stream) {
  peer_merge_kernel<<<args.heads, kPeerThreads, 0, stream>>>(args);
  return cudaGetLastError();
}

}  // namespace fa
