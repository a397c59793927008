// The peer-memory exchange of a KV-range-sharded decode (fa_peer.cu), host side.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace fa {

constexpr int kMaxPeers = 8;            // ranks of one box
constexpr int kPeerHeaderBytes = 256;   // a step counter per query head, then the stamped words
constexpr int kMaxPeerHeads = kPeerHeaderBytes / 4;

struct PeerMergeArgs {
  unsigned char* bufs[kMaxPeers];  // every rank's buffer as mapped in this process
  int rank, world, heads, head_dim;
  const float* partials;  // this rank's heads x (head_dim + 2): max, sum, o per head
  float* out;             // heads x head_dim
  unsigned* err;
};

// Bytes of each rank's buffer.
size_t peer_buffer_bytes(int world, int heads, int head_dim);
cudaError_t launch_peer_merge(const PeerMergeArgs& args, cudaStream_t stream);

}  // namespace fa
