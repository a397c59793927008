// The C ABI of include/fa_attn.h: KvCache objects in HBM, argument checks that turn the
// reference's panics into status codes, the per-call plan (chunks per row, work units) and the
// kernel launches. There is no CPU fallback: without a CUDA device every compute entry point
// returns FA_ERR_CUDA.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <queue>
#include <string>
#include <vector>

#include "fa_attn.h"
#include "fa_fmha_launch.h"
#include "fa_launch.cuh"
#include "fa_decode_tc.h"
#include "fa_relpos.h"
#include "fa_peer.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(FA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define FA_CUDA(call, what)                     \
  do {                                          \
    cudaError_t e_ = (call);                    \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

bool exact_head_dim(int d) { return d == 16 || d == 32 || d == 64 || d == 128 || d == 256; }

// Head dims with a kernel: the powers of two 16..256, and between 32 and 256 any whole number of
// the attention kernels' 16-byte vectors (4 f32 or 8 bf16 elements), which run on the next wider
// kernel with the lanes past the head idle (kronos' 52, iris' 80).
bool supported_head_dim(int d, int dtype) {
  if (exact_head_dim(d)) return true;
  return d > 32 && d <= 256 && d % (dtype == FA_BF16 ? 8 : 4) == 0;
}

// The split-KV kernel's D for a head_dim: itself, or the next power of two (PAD).
int kernel_dim(int d) {
  if (exact_head_dim(d)) return d;
  return d <= 64 ? 64 : d <= 128 ? 128 : 256;
}

// Per-device state: the SM count and the device error word.
struct Device {
  int sms = 0;
  unsigned* err = nullptr;
  std::atomic<int> epoch{0};  // bumped when a timeout is seen: caches re-zero their counters
};

std::mutex g_devices_mutex;
Device g_devices[64];

int device_state(int device, Device** out) {
  if (device < 0 || device >= 64) return fail(FA_ERR_ARG, "device %d out of range", device);
  std::lock_guard<std::mutex> lock(g_devices_mutex);
  Device& d = g_devices[device];
  if (d.err == nullptr) {
    int prev = 0;
    FA_CUDA(cudaGetDevice(&prev), "cudaGetDevice");
    FA_CUDA(cudaSetDevice(device), "cudaSetDevice");
    FA_CUDA(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, device),
            "cudaDeviceGetAttribute");
    FA_CUDA(cudaMalloc(&d.err, sizeof(unsigned)), "cudaMalloc(error word)");
    FA_CUDA(cudaMemset(d.err, 0, sizeof(unsigned)), "cudaMemset(error word)");
    cudaSetDevice(prev);
  }
  *out = &d;
  return FA_OK;
}

// Restores the caller's current device on scope exit.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int device) {
    if (cudaGetDevice(&prev) == cudaSuccess && prev != device) cudaSetDevice(device);
    else prev = -1;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

// A grow-only device buffer. An outgrown allocation is kept, not freed, until the buffer is
// released: a CUDA graph captured while it was current still reads and writes it on every
// replay (freeing it would leave such a graph writing freed memory), and so may kernels still in
// flight on another stream. Growth is by half again, so the kept allocations add up to at most
// twice the current one.
struct Buffer {
  void* ptr = nullptr;
  size_t bytes = 0;
  std::vector<void*> outgrown;
  int ensure(size_t want, cudaStream_t stream) {
    (void)stream;
    if (want <= bytes) return FA_OK;
    if (ptr != nullptr) outgrown.push_back(ptr);
    ptr = nullptr;
    bytes = 0;
    const size_t size = std::max<size_t>(want + want / 2, 1 << 16);
    FA_CUDA(cudaMalloc(&ptr, size), "cudaMalloc(workspace)");
    bytes = size;
    return FA_OK;
  }
  void release() {
    if (ptr != nullptr) cudaFree(ptr);
    for (void* p : outgrown) cudaFree(p);
    outgrown.clear();
    ptr = nullptr;
    bytes = 0;
  }
};

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// K/V bytes the tensor-core kernels' schedules may keep in L2 at once. Measured on B200 (126 MB
// of L2 over two dies): an 8192-row causal prefill whose every head's pairs ran at once slowed
// down past about this much K/V.
constexpr double kL2KvBudget = 48e6;

// fa_attention_batch_host's groups of sequences (their copies overlap the other group's work).
constexpr int kMaxHostGroups = 2;

// The one-tile kernel's band (FmhaArgs::band_heads): the most whole KV groups whose K/V
// (kv_bytes_per_head for each KV head) fits the L2 budget together, at least one, and a divisor
// of the KV heads so that the bands are equal.
int band_heads(int heads, int kv_heads, double kv_bytes_per_head) {
  int best = 1;
  for (int b = 2; b <= kv_heads; ++b)
    if (kv_heads % b == 0 && b * kv_bytes_per_head <= kL2KvBudget) best = b;
  return best * (heads / kv_heads);
}

// The schedule of a bf16 full-mask call's units (query head, pair of 128-row query tiles) over
// `sms` SMs: the first `whole` units run as one CTA each and every later unit as `splits` pieces
// over equal shares of its `kv_tiles` key tiles. Units whose count is not a multiple of the SM
// count leave the last wave partly idle; cutting the units after the last full wave (or the last
// two) into shorter pieces fills it. Cost model, in units of one whole unit's time: a wave of
// whole units costs 1, a wave of pieces 1 / splits plus a fixed cost per CTA of about 16 key
// tiles (start, pipeline fill, partials and merge: measured on B200 with 256-tile units, where
// a whole unit is about 500 us and splitting one in two costs about 30 us more in all). A split
// is taken when it saves at least 2%.
void plan_full_split(int64_t units, int sms, int kv_tiles, int64_t* whole, int* splits) {
  *whole = units;
  *splits = 1;
  if (units <= 0 || sms <= 0 || units % sms == 0) return;
  const int64_t full = units / sms;
  const double unsplit = double(full + 1);
  const double fixed = 16.0 / std::max(kv_tiles, 1);
  double best = unsplit;
  for (int64_t lead_waves = std::max<int64_t>(full - 1, 0); lead_waves <= full; ++lead_waves) {
    const int64_t tail = units - lead_waves * sms;
    for (int s = 2; s <= fa::kFmhaMaxSplits && kv_tiles >= 4 * s; ++s) {
      const double cost = double(lead_waves) + double((tail * s + sms - 1) / sms) * (1.0 / s + fixed);
      if (cost < best) {
        best = cost;
        *whole = lead_waves * sms;
        *splits = s;
      }
    }
  }
  if (*splits > 1 && best >= 0.98 * unsplit) {
    *whole = units;
    *splits = 1;
  }
}

// Partials and arrival counters of split full-mask calls, one set per (device, stream): calls on
// one stream run in order, so they can share it; calls on different streams get their own.
struct SplitWork {
  Buffer partials;
  Buffer counters;  // zero between launches (the last piece of a unit resets its counter)
  int counters_epoch = -1;
};
std::mutex g_split_mutex;
std::map<std::pair<int, cudaStream_t>, SplitWork> g_split_work;
// The same for the f32 full-mask calls that run on the split-KV kernel (queries, partials).
std::map<std::pair<int, cudaStream_t>, SplitWork> g_full_work;
constexpr size_t kMaxSplitBytes = size_t(512) << 20;

}  // namespace

struct fa_kvcache {
  int layers, heads, kv_heads, head_dim, capacity, dtype, device;
  void* keys = nullptr;
  void* values = nullptr;
  Device* dev = nullptr;
  Buffer work;       // queries and partials
  Buffer staging;    // fa_attention_host's device copies of the host rows
  Buffer counters;   // arrival counters (kept zero between launches)
  Buffer tc_maps;    // bf16, head_dim 128 or 256: TMA maps over the keys and values (tensor-core
                     // decode)
  Buffer proj_work;      // the projections' partial sums (and the tensor-core one's projected rows)
  Buffer proj_counters;  // and its arrival counters (kept zero between launches)
  Buffer io;             // fa_attention_batch_host's device copies of the host rows
  cudaStream_t copy_stream = nullptr;  // and its copies, beside the caller's stream
  cudaStream_t side_stream = nullptr;  // and its odd groups, concurrent with the even ones
  cudaEvent_t io_events[2 * kMaxHostGroups + 1] = {};  // rows in, attention done (per group),
                                                       // the side stream's end
  int counters_epoch = 0;
  int proj_epoch = -1;
  size_t elem() const { return dtype == FA_F32 ? 4 : 2; }
  int64_t layer_elems() const { return int64_t(kv_heads) * capacity * head_dim; }
};

namespace {

int check_cache(const fa_kvcache* cache) {
  if (cache == nullptr) return fail(FA_ERR_ARG, "null cache");
  return FA_OK;
}

// Whether the kernels on `device` may address `ptr`: memory of that device, managed memory, or
// pinned host memory mapped into the device's address space. Another device's memory and
// pageable host memory are rejected here: a kernel given them faults.
int check_ptr(const void* ptr, int device, const char* what) {
  if (ptr == nullptr) return FA_OK;
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, ptr) != cudaSuccess) {
    cudaGetLastError();
    return fail(FA_ERR_ARG, "%s is not memory CUDA knows", what);
  }
  if (attr.type == cudaMemoryTypeDevice) {
    if (attr.device != device)
      return fail(FA_ERR_ARG, "%s is on device %d, the call runs on device %d", what, attr.device,
                  device);
    return FA_OK;
  }
  if (attr.type == cudaMemoryTypeManaged) return FA_OK;
  if (attr.type == cudaMemoryTypeHost && attr.devicePointer != nullptr) return FA_OK;
  return fail(FA_ERR_ARG, "%s is pageable host memory; device memory is needed here", what);
}

#define FA_PTR(ptr, device) \
  do {                      \
    if (int rc_ = check_ptr((ptr), (device), #ptr)) return rc_; \
  } while (0)

int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) d = 0;
  return d;
}

// Host rows (`stride` floats apart) to `width`-float device rows: one linear copy when the rows
// are contiguous (the 2D form's per-row transfers cost more), else a pitched one.
cudaError_t rows_to_device(float* dst, int64_t width, const float* src, int64_t stride,
                           int64_t rows, cudaStream_t s) {
  if (stride == width)
    return cudaMemcpyAsync(dst, src, size_t(rows * width) * 4, cudaMemcpyHostToDevice, s);
  return cudaMemcpy2DAsync(dst, size_t(width) * 4, src, size_t(stride) * 4, size_t(width) * 4,
                           size_t(rows), cudaMemcpyHostToDevice, s);
}

int ensure_counters(fa_kvcache* c, size_t n, cudaStream_t stream) {
  const size_t want = n * sizeof(int);
  const int epoch = c->dev->epoch.load();
  if (want <= c->counters.bytes && epoch == c->counters_epoch) return FA_OK;
  if (int rc = c->counters.ensure(want, stream)) return rc;
  FA_CUDA(cudaMemsetAsync(c->counters.ptr, 0, c->counters.bytes, stream), "cudaMemsetAsync(counters)");
  c->counters_epoch = epoch;
  return FA_OK;
}

// Checks a span against the cache (Transformer::run, transformer.rs:329-341; Mask::Groups's
// ends, transformer.rs:107-110) and copies its Groups ends.
int check_span(const fa_kvcache* c, const fa_span* span, std::vector<int>* ends) {
  if (span == nullptr) return fail(FA_ERR_ARG, "null span");
  if (span->rows < 0 || span->first < 0) return fail(FA_ERR_ARG, "negative span");
  const fa_mask& m = span->mask;
  if (m.kind < FA_MASK_CAUSAL || m.kind > FA_MASK_GROUPS)
    return fail(FA_ERR_ARG, "mask kind %d", m.kind);
  const int64_t end = int64_t(span->first) + span->rows;
  if (m.kind == FA_MASK_WINDOW && m.window < 1) return fail(FA_ERR_ARG, "window %d", m.window);
  const int64_t reach = m.kind == FA_MASK_WINDOW ? int64_t(m.window) + span->rows : end;
  if (reach > c->capacity)
    return fail(FA_ERR_CAPACITY, "the cache holds every key the span sees: %lld > capacity %d",
                (long long)reach, c->capacity);
  ends->clear();
  if (m.kind == FA_MASK_GROUPS) {
    if (m.n_ends < 1 || m.ends == nullptr || m.n_ends > fa::kMaxEnds)
      return fail(FA_ERR_ARG, "Groups needs 1..%d ends", fa::kMaxEnds);
    if (m.state < 0 || m.state > end) return fail(FA_ERR_ARG, "Groups state %d", m.state);
    for (int i = 0; i < m.n_ends; ++i) {
      if (m.ends[i] <= (i == 0 ? m.state - 1 : m.ends[i - 1]) || m.ends[i] > end)
        return fail(FA_ERR_ARG, "Groups ends must rise after the state and end by the call's end");
      ends->push_back(m.ends[i]);
    }
    if (ends->back() != end) return fail(FA_ERR_ARG, "the last group ends with the call");
  }
  return FA_OK;
}

float query_scale(int head_dim) {
  return float((1.0 / std::sqrt(double(head_dim))) * 1.4426950408889634);
}

int heads_per_cta(int group) {
  if (group >= 8) return 8;
  if (group >= 4) return group == 4 ? 4 : 8;
  return group;  // 1, 2 or 3 -> 1, 2, 4
}

int pow2_heads(int group) {
  const int g = heads_per_cta(group);
  return g == 3 ? 4 : g;
}

// Work units wanted per launch: FA_DECODE_WAVES waves of the split-KV kernel's resident CTAs.
#ifndef FA_DECODE_WAVES
#define FA_DECODE_WAVES 4
#endif
int target_units(const Device* dev) {
  return std::max(dev->sms, 1) * FA_DECODE_MIN_CTAS * FA_DECODE_WAVES;
}

struct Plan {
  int g = 1, hgroups = 1, kv_groups = 1, chunks = 1;
  int cluster = 0;  // > 1: a row's chunks form a thread-block cluster and merge in shared memory
};

#ifndef FA_DECODE_CLUSTER
#define FA_DECODE_CLUSTER 1
#endif
#ifndef FA_SPAN_MIN_CHUNK_TILES
#define FA_SPAN_MIN_CHUNK_TILES 16
#endif

int attend_resident_d(int head_dim, const fa::AttendLaunch& launch) {
  fa::AttendLaunch l = launch;
  l.pad = kernel_dim(head_dim) != head_dim;
  switch (kernel_dim(head_dim)) {
    case 16: return fa::attend_resident<16>(l);
    case 32: return fa::attend_resident<32>(l);
    case 64: return fa::attend_resident<64>(l);
    case 128: return fa::attend_resident<128>(l);
    case 256: return fa::attend_resident<256>(l);
    default: return 0;
  }
}

// The chunk count, at most p.chunks, that streams a span's keys in the least time when the CTAs
// run in waves of the SMs' resident slots: a last wave that is mostly empty streams at a fraction
// of the rate (fewer loads in flight per SM) for as long as a full one, so the cost of c chunks
// is waves(c) / c (waves times each chunk's share of the keys); the largest count of least cost.
// A GPU's share of C4 over 2 GPUs (65537 keys, 8 KV heads, 444 slots): 128 chunks = 2.3 waves
// -> 111 chunks, 2 waves; over 4 GPUs 64 -> 55 chunks, one wave.
int whole_waves(const fa_kvcache* c, int rows, const Plan& p) {
  fa::AttendLaunch l{};
  l.kt = c->dtype == FA_F32 ? fa::kKtF32 : fa::kKtBf16;
  l.g = p.g;
  l.batch = false;
  const int resident = attend_resident_d(c->head_dim, l);
  if (resident <= 0) return p.chunks;
  const int64_t slots = int64_t(c->dev->sms) * resident;
  const int64_t per_chunk = int64_t(rows) * p.kv_groups;
  auto cost = [&](int ch) { return double((per_chunk * ch + slots - 1) / slots) / ch; };
  int best = p.chunks;
  double best_cost = cost(best);
  for (int ch = p.chunks - 1; ch >= 1; --ch) {
    if (cost(ch) < best_cost * (1.0 - 1e-9)) {
      best_cost = cost(ch);
      best = ch;
    }
  }
  return best;
}

Plan plan_span(const fa_kvcache* c, int rows, int max_keys, bool split_small = true) {
  Plan p;
  const int group = c->heads / c->kv_heads;
  p.g = pow2_heads(group);
  const int tile = fa::tile_keys(kernel_dim(c->head_dim), c->dtype == FA_F32 ? fa::kKtF32 : fa::kKtBf16);
  const int max_chunks = std::max(1, (max_keys + tile - 1) / tile);
  // A launch too small for a CTA on every SM (a short decode, C1's 1025 keys) splits each KV
  // head's query heads over more CTAs: each re-reads the KV head, from L2 at these sizes.
  auto units = [&](int g) {
    return int64_t(rows) * c->kv_heads * ((group + g - 1) / g) * max_chunks;
  };
  while (split_small && p.g > 2 && units(p.g / 2) <= c->dev->sms) p.g /= 2;
  p.hgroups = (group + p.g - 1) / p.g;
  p.kv_groups = c->kv_heads * p.hgroups;
  const int want = (target_units(c->dev) + rows * p.kv_groups - 1) / std::max(rows * p.kv_groups, 1);
  p.chunks = std::min(max_chunks, std::max(1, want));
  // A short row (at most four tiles per CTA of a cluster) in a launch that fits on the SMs has
  // its chunks as one cluster, merged in shared memory (no partials through HBM, no arrival
  // counter): the latency of a short decode (C1's 1025 keys).
  const int clustered = std::min(p.chunks, fa::kMaxClusterChunks);
  if (split_small && FA_DECODE_CLUSTER && p.chunks > 1 &&
      max_chunks <= 4 * fa::kMaxClusterChunks &&
      int64_t(rows) * p.kv_groups * clustered <= c->dev->sms) {
    p.chunks = clustered;
    p.cluster = clustered;
  } else {
    // Otherwise a chunk spans at least FA_SPAN_MIN_CHUNK_TILES tiles: a CTA's fixed cost (its
    // start, the query, its partial and the arrival) outweighs a few tiles' streaming. Measured
    // on B200 for one row over 16384 keys of 8 f32 KV heads (a GPU's share of C4 over 8 GPUs):
    // 37 vs 63 us against 3.5-tile chunks; 131073 keys keep their 148 chunks.
    p.chunks = std::min(p.chunks, std::max(1, max_chunks / FA_SPAN_MIN_CHUNK_TILES));
    p.chunks = whole_waves(c, rows, p);
  }
  return p;
}

// Workspace layout of one call: rotated queries, chunk partials (o then max/sum).
struct Work {
  float* q = nullptr;
  float* part_o = nullptr;
  float* part_ml = nullptr;
};

int ensure_work(fa_kvcache* c, size_t q_floats, size_t part_slots, size_t unused,
                cudaStream_t stream, Work* w) {
  (void)unused;
  const size_t q_bytes = align_up(q_floats * 4, 256);
  // a chunk's partial output is the kernel's D wide (kernel_dim: a padded head_dim's kernel)
  const size_t o_bytes = align_up(part_slots * kernel_dim(c->head_dim) * 4, 256);
  const size_t ml_bytes = align_up(part_slots * 2 * 4, 256);
  if (int rc = c->work.ensure(q_bytes + o_bytes + ml_bytes, stream)) return rc;
  unsigned char* base = static_cast<unsigned char*>(c->work.ptr);
  w->q = reinterpret_cast<float*>(base);
  w->part_o = reinterpret_cast<float*>(base + q_bytes);
  w->part_ml = reinterpret_cast<float*>(base + q_bytes + o_bytes);
  return FA_OK;
}

void fill_common(fa::AttendCommon* a, const fa_kvcache* c, const Plan& p) {
  a->heads = c->heads;
  a->kv_heads = c->kv_heads;
  a->group = c->heads / c->kv_heads;
  a->hgroups = p.hgroups;
  a->kv_stride = int64_t(c->capacity) * c->head_dim;
  a->key_stride = c->head_dim;
  a->q_scale = query_scale(c->head_dim);
  a->err = c->dev->err;
  a->dh = c->head_dim;
}

cudaError_t launch_attend_d(int head_dim, const fa::AttendLaunch& launch, cudaStream_t stream) {
  fa::AttendLaunch l = launch;
  l.pad = kernel_dim(head_dim) != head_dim;
  switch (kernel_dim(head_dim)) {
    case 16: return fa::launch_attend<16>(l, stream);
    case 32: return fa::launch_attend<32>(l, stream);
    case 64: return fa::launch_attend<64>(l, stream);
    case 128: return fa::launch_attend<128>(l, stream);
    case 256: return fa::launch_attend<256>(l, stream);
    default: return cudaErrorInvalidValue;
  }
}

const unsigned char* layer_ptr(const fa_kvcache* c, const void* base, int layer) {
  return static_cast<const unsigned char*>(base) + size_t(layer) * c->layer_elems() * c->elem();
}

// The plan of a span over a cache: the largest key count of its rows decides the chunks.
Plan plan_for_span(const fa_kvcache* c, const fa_span* span, const std::vector<int>& ends) {
  int max_keys = 0;
  for (int r = 0; r < span->rows; ++r) {
    fa::Runs runs = fa::mask_runs(span->mask.kind, span->mask.window, span->mask.state,
                                  int(ends.size()), ends.data(), span->first + r,
                                  span->first + span->rows);
    max_keys = std::max(max_keys, runs.n0 + runs.n1);
  }
  return plan_span(c, std::max(span->rows, 1), max_keys);
}

// Whether a batch of one-row decodes runs on the tensor cores: bf16 caches of head_dim 128 or 256
// with their TMA maps, at most 16 query heads per KV head, and every row's keys one run of cache
// slots without a ring wrap (a window that wraps, or Groups' two runs, decode on the CUDA cores).
#ifndef FA_DECODE_TC
#define FA_DECODE_TC 1
#endif
bool decode_on_tensor_cores(fa_kvcache* const* caches, const std::vector<fa::Runs>& runs,
                            int batch) {
  if (!FA_DECODE_TC) return false;
  const fa_kvcache* c0 = caches[0];
  if (c0->dtype != FA_BF16 || (c0->head_dim != 128 && c0->head_dim != 256) ||
      c0->heads / c0->kv_heads > fa::kDtcN)
    return false;
  for (int i = 0; i < batch; ++i) {
    const fa_kvcache* c = caches[i];
    if (c->tc_maps.ptr == nullptr || runs[i].n1 != 0 || runs[i].n0 < 1 ||
        runs[i].b0 + runs[i].n0 > c->capacity)
      return false;
  }
  return true;
}

// The chunking of a tensor-core decode: chunks of a common length (a multiple of 128 keys), about
// FA_DTC_UNITS (row, KV head, chunk) units per CTA (measured best: 1, the fewest unit ends and
// chunk merges; the schedule balances whole rows), at most kDtcMaxUnits a launch. Measured on
// B200 over a GPU's share of C3 (bf16) at 1, 2, 4 and 8 GPUs, 1..8 units a CTA: 1 is fastest at
// 64, 32 and 16 sequences (181 / 101 / 62 us; 8 units: 224 / 139 / 102 us) and within 2 % of 2
// units at 8 sequences (43.6 vs 42.9 us).
#ifndef FA_DTC_UNITS
#define FA_DTC_UNITS 1
#endif
struct DtcPlan {
  int64_t chunk_keys = 0;
  int64_t slots = 0;  // partial chunk slots of every row (heads each)
  std::vector<int> chunks, part_base;
};

DtcPlan plan_decode_tc(const fa_kvcache* c0, const std::vector<fa::Runs>& runs, int batch) {
  DtcPlan p;
  int64_t total_keys = 0;
  for (int i = 0; i < batch; ++i) total_keys += runs[i].n0;
  const int sms = std::max(1, std::min(c0->dev->sms, fa::kDtcMaxCtas));
  for (int64_t want = int64_t(sms) * FA_DTC_UNITS;; want = want * 3 / 4) {
    p.chunk_keys = (total_keys * c0->kv_heads + want - 1) / want;
    p.chunk_keys = std::max<int64_t>(fa::kDtcKeys, (p.chunk_keys + fa::kDtcKeys - 1) / fa::kDtcKeys * fa::kDtcKeys);
    int64_t units = 0;
    for (int i = 0; i < std::min(batch, fa::kMaxBatchRows); ++i)
      units += c0->kv_heads * ((runs[i].n0 + p.chunk_keys - 1) / p.chunk_keys);
    if (units <= fa::kDtcMaxUnits || want <= 1) break;
  }
  p.chunks.resize(batch);
  p.part_base.resize(batch);
  for (int i = 0; i < batch; ++i) {
    p.chunks[i] = int((runs[i].n0 + p.chunk_keys - 1) / p.chunk_keys);
    p.part_base[i] = int(p.slots);
    p.slots += p.chunks[i];
  }
  return p;
}

// A span's rows as the tensor-core decode's batch rows (each row its keys from the mask), when
// the span decodes there: rows of one run of cache slots each.
bool span_decode_tc(fa_kvcache* c, const fa_span* span, const std::vector<int>& ends,
                    std::vector<fa::Runs>* runs) {
  runs->resize(span->rows);
  for (int r = 0; r < span->rows; ++r)
    (*runs)[r] = fa::mask_runs(span->mask.kind, span->mask.window, span->mask.state,
                               int(ends.size()), ends.data(), span->first + r,
                               span->first + span->rows);
  std::vector<fa_kvcache*> caches(span->rows, c);
  return span->rows > 0 && decode_on_tensor_cores(caches.data(), *runs, span->rows);
}

// The tensor-core decode of a batch (persistent CTAs, one per SM; `given`: the caller's workspace,
// sized for plan_decode_tc's slots).
int attend_batch_tc(fa_kvcache* const* caches, const std::vector<fa::Runs>& runs, int batch,
                    int layer, const float* q, int64_t q_stride, float* out, int64_t out_stride,
                    cudaStream_t s, const Work* given = nullptr) {
  fa_kvcache* c0 = caches[0];
  const int sms = std::max(1, std::min(c0->dev->sms, fa::kDtcMaxCtas));
  const DtcPlan plan = plan_decode_tc(c0, runs, batch);
  const int64_t chunk_keys = plan.chunk_keys;
  const std::vector<int>& chunks = plan.chunks;
  const std::vector<int>& part_base = plan.part_base;
  Work w;
  if (given != nullptr) w = *given;  // sized by the caller (tc_decode_slots)
  else if (int rc = ensure_work(c0, 0, size_t(plan.slots) * c0->heads, 0, s, &w)) return rc;
  if (int rc = ensure_counters(c0, size_t(batch) * c0->kv_heads, s)) return rc;
  for (int first = 0; first < batch; first += fa::kMaxBatchRows) {
    const int n = std::min(batch - first, fa::kMaxBatchRows);
    fa::DtcArgs a{};
    a.heads = c0->heads;
    a.kv_heads = c0->kv_heads;
    a.group = c0->heads / c0->kv_heads;
    a.n_rows = n;
    a.chunk_keys = int(chunk_keys);
    a.q = q + int64_t(first) * q_stride;
    a.q_stride = q_stride;
    a.scale_log2 = query_scale(c0->head_dim);
    a.out = out + int64_t(first) * out_stride;
    a.out_stride = out_stride;
    a.part_o = w.part_o;
    a.part_ml = w.part_ml;
    a.counters = static_cast<int*>(c0->counters.ptr) + int64_t(first) * c0->kv_heads;
    a.err = c0->dev->err;
    int units = 0;
    for (int i = 0; i < n; ++i) {
      const fa_kvcache* c = caches[first + i];
      fa::DtcRow& r = a.rows[i];
      r.kmap = c->tc_maps.ptr;
      r.vmap = static_cast<const unsigned char*>(c->tc_maps.ptr) + 128;
      r.z0 = layer * c->kv_heads;
      r.b0 = runs[first + i].b0;
      r.n = runs[first + i].n0;
      r.chunks = chunks[first + i];
      r.unit_begin = units;
      r.part_base = part_base[first + i];
      units += c0->kv_heads * r.chunks;
    }
    a.n_units = units;
    // Longest processing time first: the units by tiles, longest first (a counting sort), each
    // to the least loaded CTA (a heap); each CTA's list keeps that order.
    const int ctas = std::min(units, sms);
    const int max_tiles = int((chunk_keys + fa::kDtcKeys - 1) / fa::kDtcKeys);
    std::vector<int> unit_tiles(units), count(max_tiles + 2, 0);
    for (int i = 0, u = 0; i < n; ++i) {
      const int64_t nk = a.rows[i].n;
      for (int k = 0; k < c0->kv_heads; ++k)
        for (int ch = 0; ch < a.rows[i].chunks; ++ch, ++u) {
          const int64_t keys = std::min<int64_t>(nk, int64_t(ch + 1) * chunk_keys) - int64_t(ch) * chunk_keys;
          unit_tiles[u] = int((keys + fa::kDtcKeys - 1) / fa::kDtcKeys);
          ++count[max_tiles - unit_tiles[u]];
        }
    }
    for (int t = 1; t <= max_tiles + 1; ++t) count[t] += count[t - 1];
    std::vector<int> sorted(units);
    for (int u = units - 1; u >= 0; --u) sorted[--count[max_tiles - unit_tiles[u]]] = u;
    using Load = std::pair<int64_t, int>;  // (tiles assigned, CTA)
    std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap;
    for (int c = 0; c < ctas; ++c) heap.push({0, c});
    std::vector<int> owner(units), per_cta(ctas + 1, 0);
    for (int u : sorted) {
      Load l = heap.top();
      heap.pop();
      owner[u] = l.second;
      ++per_cta[l.second + 1];
      l.first += unit_tiles[u] + 1;  // a unit's own start and end cost about a tile
      heap.push(l);
    }
    for (int c = 0; c < ctas; ++c) per_cta[c + 1] += per_cta[c];
    for (int c = 0; c <= ctas; ++c) a.cta_first[c] = uint16_t(per_cta[c]);
    for (int u : sorted) a.order[per_cta[owner[u]]++] = uint16_t(u);
    cudaError_t e = fa::launch_decode_tc(a, c0->head_dim, ctas, s);
    if (e != cudaSuccess) return cuda_fail(e, "tensor-core decode launch");
  }
  return FA_OK;
}

// The attention of a span's rows over the cache, queries already rotated and scaled in q;
// `w` holds the partials of `p`.
int attend_rows(fa_kvcache* c, int layer, const fa_span* span, const std::vector<int>& ends,
                const Plan& p, const Work& w, const float* q, int64_t q_stride, float* out,
                int64_t out_stride, float* partial_out, cudaStream_t stream) {
  const int rows = span->rows;
  if (rows == 0) return FA_OK;
  if (int rc = ensure_counters(c, size_t(rows) * p.kv_groups, stream)) return rc;
  fa::SpanArgs args{};
  fill_common(&args.c, c, p);
  args.c.q = q;
  args.c.q_stride = q_stride;
  args.c.out = out;
  args.c.out_stride = out_stride;
  args.c.partial_out = partial_out;
  args.c.part_o = w.part_o;
  args.c.part_ml = w.part_ml;
  args.c.counters = static_cast<int*>(c->counters.ptr);
  args.k = layer_ptr(c, c->keys, layer);
  args.v = layer_ptr(c, c->values, layer);
  args.capacity = c->capacity;
  args.rows = rows;
  args.first = span->first;
  args.end = span->first + rows;
  args.kind = span->mask.kind;
  args.window = span->mask.window;
  args.state = span->mask.state;
  args.n_ends = int(ends.size());
  args.chunks = p.chunks;
  args.c.cluster = p.cluster;
  args.rows_per_image = rows;
  args.keys_per_image = 0;
  for (size_t i = 0; i < ends.size(); ++i) args.ends[i] = ends[i];
  fa::AttendLaunch l{c->dtype == FA_F32 ? fa::kKtF32 : fa::kKtBf16, p.g, false, &args, nullptr,
                     rows * p.kv_groups * p.chunks};
  cudaError_t e = launch_attend_d(c->head_dim, l, stream);
  if (e != cudaSuccess) return cuda_fail(e, "attend launch");
  return FA_OK;
}

// Rows from which a span goes to the tensor-core kernel (below it the split-KV kernel, which
// needs no 128-row tiles, is as fast).
#ifndef FA_TC_MIN_ROWS
#define FA_TC_MIN_ROWS 64
#endif
constexpr int kFmhaMinRows = FA_TC_MIN_ROWS;

// Whether a span over the cache runs on the tcgen05 kernel: head_dim 64 or 128, enough rows,
// and no key position wraps the cache's ring (a causal or full span never does; a window span
// does once first + rows passes the capacity).
bool span_on_tensor_cores(const fa_kvcache* c, const fa_span* span) {
  if (span->rows < kFmhaMinRows) return false;
  if (!fa::fmha_supported(c->dtype == FA_BF16, c->head_dim)) return false;
  return int64_t(span->first) + span->rows <= c->capacity;
}

// The tcgen05 attention of a span's rows over the cache; q holds the rotated queries in the
// cache's element type (rows x q_stride elements, heads x head_dim each).
int attend_rows_tc(fa_kvcache* c, int layer, const fa_span* span, const std::vector<int>& ends,
                   const void* q, int64_t q_stride, float* out, int64_t out_stride,
                   cudaStream_t stream) {
  fa::FmhaArgs a{};
  a.heads = c->heads;
  a.kv_heads = c->kv_heads;
  a.group = c->heads / c->kv_heads;
  a.rows = span->rows;
  a.images = 1;
  a.q_tiles = (span->rows + 127) / 128;
  a.first = span->first;
  a.end = span->first + span->rows;
  a.kind = span->mask.kind;
  a.window = span->mask.window;
  a.state = span->mask.state;
  a.n_ends = int(ends.size());
  for (size_t i = 0; i < ends.size(); ++i) a.ends[i] = ends[i];
  a.q_row_base_per_image = 0;
  a.kv_row_base_per_image = 0;
  a.kv_layer_base = layer * c->kv_heads;
  a.scale_log2 = query_scale(c->head_dim);
  a.out = out;
  a.out_stride = out_stride;
  a.out_bf16 = 0;
  a.err = c->dev->err;
  // A causal span whose rows see from a few keys to several times as many runs its heaviest
  // pairs first across heads, when the K/V it reads fits well inside L2 (every head's pairs run
  // at once in that order). Measured on B200: an 8192-row causal prefill from position 0 (32/8
  // heads x 128, bf16 cache).
  const double kv_head_bytes = 2.0 * double(a.end) * c->head_dim * c->elem();
  a.pair_major = a.kind == FA_MASK_CAUSAL && span->first < span->rows &&
                 c->kv_heads * kv_head_bytes <= kL2KvBudget;
  a.band_heads = band_heads(c->heads, c->kv_heads, kv_head_bytes);
  fa::FmhaLaunch l{c->dtype == FA_BF16 ? 1 : 0, c->head_dim, q, uint64_t(span->rows),
                   uint64_t(c->heads), uint64_t(q_stride), uint64_t(c->head_dim), c->keys,
                   c->values, uint64_t(c->capacity), uint64_t(c->layers) * c->kv_heads,
                   uint64_t(c->head_dim), uint64_t(c->capacity) * c->head_dim, a};
  cudaError_t e = fa::launch_fmha(l, stream);
  if (e != cudaSuccess) return cuda_fail(e, "tensor-core attention launch");
  return FA_OK;
}

int rope_rows(fa_kvcache* c, int layer, const fa_span* span, int rope, const float* angles,
              const fa_head_norm* norm, const float* qkv, int64_t qkv_stride, float* q_out,
              int64_t q_out_stride, float q_scale, bool keep, cudaStream_t stream,
              bool q_out_bf16 = false, int gate_heads = 0, int rotary_dim = 0) {
  if (span->rows == 0) return FA_OK;
  fa::RopeArgs a{};
  a.heads = c->heads;
  a.kv_heads = c->kv_heads;
  a.head_dim = c->head_dim;
  a.gate_heads = gate_heads;
  a.rotary_dim = rotary_dim;
  a.rope = rope;
  a.n_rows = span->rows;
  a.qkv = qkv;
  a.qkv_stride = qkv_stride;
  a.angles = angles;
  a.q_norm = norm ? norm->q_norm : nullptr;
  a.k_norm = norm ? norm->k_norm : nullptr;
  a.eps = norm ? norm->eps : 0.0f;
  a.q_out = q_out;
  a.q_out_stride = q_out_stride;
  a.q_scale = q_scale;
  a.q_out_bf16 = q_out_bf16 ? 1 : 0;
  a.keep = keep ? 1 : 0;
  a.batch = 0;
  a.first = span->first;
  a.keep_rows[0].k = const_cast<unsigned char*>(layer_ptr(c, c->keys, layer));
  a.keep_rows[0].v = const_cast<unsigned char*>(layer_ptr(c, c->values, layer));
  a.keep_rows[0].capacity = c->capacity;
  cudaError_t e = fa::launch_rope(c->dtype == FA_F32 ? fa::kKtF32 : fa::kKtBf16, a, stream);
  if (e != cudaSuccess) return cuda_fail(e, "rope launch");
  return FA_OK;
}

int check_layer(const fa_kvcache* c, int layer) {
  if (layer < 0 || layer >= c->layers)
    return fail(FA_ERR_SHAPE, "layer %d of a %d-layer cache", layer, c->layers);
  return FA_OK;
}

int check_rope(int rope, const float* angles) {
  if (rope < FA_ROPE_NONE || rope > FA_ROPE_INTERLEAVED) return fail(FA_ERR_ARG, "rope %d", rope);
  if (rope != FA_ROPE_NONE && angles == nullptr) return fail(FA_ERR_ARG, "RoPE without angles");
  return FA_OK;
}

// Rotary::new + spatially_scaled (rotary.rs:117-168): the frequencies and the axis of each.
int rotary_frequencies(const fa_rotation* r, int head_dim, std::vector<float>* inv_freq,
                       std::vector<int>* axes) {
  const int half = head_dim / 2;
  auto inv = [&](int dims, std::vector<float>* out) {
    out->resize(dims / 2);
    for (int i = 0; i < dims / 2; ++i)
      (*out)[i] = 1.0f / std::pow(r->base, float(2 * i) / float(dims));
  };
  auto sections = [&](const int32_t* s) {
    if (s[0] < 0 || s[1] < 0 || s[2] < 0 || s[0] + s[1] + s[2] != half) return false;
    axes->clear();
    for (int a = 0; a < 3; ++a) axes->insert(axes->end(), s[a], a);
    return true;
  };
  axes->assign(half, 0);
  switch (r->kind) {
    case FA_ROT_SEQUENCE:
      inv(head_dim, inv_freq);
      break;
    case FA_ROT_LINEAR:
      if (r->params[0] <= 0) return fail(FA_ERR_ARG, "Linear factor %d", r->params[0]);
      inv(head_dim, inv_freq);
      for (auto& f : *inv_freq) f = f / float(r->params[0]);
      break;
    case FA_ROT_PARTIAL:
      inv(head_dim, inv_freq);
      for (int i = std::max(0, r->params[0]); i < half; ++i) (*inv_freq)[i] = 0.0f;
      break;
    case FA_ROT_MULTIMODAL:
      inv(head_dim, inv_freq);
      if (!sections(r->params)) return fail(FA_ERR_ARG, "sections do not cover half a head");
      break;
    case FA_ROT_AXES:
    case FA_ROT_GRID: {
      const int32_t grid[3] = {0, half / 2, half / 2};
      const int32_t* s = r->kind == FA_ROT_GRID ? grid : r->params;
      if (!sections(s)) return fail(FA_ERR_ARG, "sections do not cover half a head");
      inv_freq->clear();
      for (int a = 0; a < 3; ++a) {
        std::vector<float> part;
        inv(2 * s[a], &part);
        inv_freq->insert(inv_freq->end(), part.begin(), part.end());
      }
      break;
    }
    case FA_ROT_MULTIMODAL_INTERLEAVED:
      inv(head_dim, inv_freq);
      for (int i = 0; i < half; ++i) {
        const int m = i % 3;
        (*axes)[i] = (m == 1 && i < 3 * r->params[1]) ? 1 : (m == 2 && i < 3 * r->params[2]) ? 2 : 0;
      }
      break;
    default:
      return fail(FA_ERR_ARG, "rotation kind %d", r->kind);
  }
  for (int i = 0; i < half; ++i)
    if ((*axes)[i] != 0) (*inv_freq)[i] = (*inv_freq)[i] * r->spatial_scale;
  return FA_OK;
}

}  // namespace

extern "C" {

const char* fa_last_error(void) { return g_last_error.c_str(); }

int fa_capabilities(int32_t* flags, int32_t* head_dims, int32_t max_head_dims,
                    int32_t* n_head_dims) {
  static const int32_t dims[] = {16, 32, 64, 128, 256};
  if (flags) *flags = 1 | 2 | (fa::fmha_supported(1, 128) ? 4 : 0) | 8;
  const int n = int(sizeof dims / sizeof dims[0]);
  if (head_dims)
    for (int i = 0; i < n && i < max_head_dims; ++i) head_dims[i] = dims[i];
  if (n_head_dims) *n_head_dims = n;
  return FA_OK;
}

int fa_kvcache_create(int32_t layers, int32_t heads, int32_t kv_heads, int32_t head_dim,
                      int32_t capacity, int32_t dtype, int32_t device, fa_kvcache** out) {
  if (out == nullptr) return fail(FA_ERR_ARG, "null out");
  *out = nullptr;
  if (layers < 1 || heads < 1 || kv_heads < 1 || capacity < 1)
    return fail(FA_ERR_ARG, "a cache of %d layers, %d heads, %d kv heads, capacity %d", layers,
                heads, kv_heads, capacity);
  if (heads % kv_heads != 0)
    return fail(FA_ERR_SHAPE, "%d heads over %d KV heads", heads, kv_heads);
  if (!supported_head_dim(head_dim, dtype)) return fail(FA_ERR_UNSUPPORTED, "head_dim %d", head_dim);
  if (dtype != FA_F32 && dtype != FA_BF16) return fail(FA_ERR_ARG, "dtype %d", dtype);
  Device* dev = nullptr;
  if (int rc = device_state(device, &dev)) return rc;
  DeviceGuard guard(device);
  auto* c = new fa_kvcache();
  c->layers = layers;
  c->heads = heads;
  c->kv_heads = kv_heads;
  c->head_dim = head_dim;
  c->capacity = capacity;
  c->dtype = dtype;
  c->device = device;
  c->dev = dev;
  const size_t bytes = size_t(layers) * c->layer_elems() * c->elem();
  cudaError_t e = cudaMalloc(&c->keys, bytes);
  if (e == cudaSuccess) e = cudaMalloc(&c->values, bytes);
  if (e == cudaSuccess) e = cudaMemset(c->keys, 0, bytes);
  if (e == cudaSuccess) e = cudaMemset(c->values, 0, bytes);
  if (e != cudaSuccess) {
    fa_kvcache_destroy(c);
    return cuda_fail(e, "cache allocation");
  }
  if (dtype == FA_BF16 && (head_dim == 128 || head_dim == 256)) {
    // TMA maps of the keys and values for the tensor-core decode, made once: [layers x kv heads]
    // [capacity][head_dim] (a cache that cannot have them decodes on the CUDA cores)
    alignas(64) unsigned char maps[256];
    const uint64_t z_stride = uint64_t(capacity) * head_dim * 2;
    if (fa::encode_cache_map_bf16(maps, c->keys, uint64_t(head_dim), uint64_t(capacity),
                                  uint64_t(layers) * kv_heads, z_stride) &&
        fa::encode_cache_map_bf16(maps + 128, c->values, uint64_t(head_dim), uint64_t(capacity),
                                  uint64_t(layers) * kv_heads, z_stride)) {
      e = cudaMalloc(&c->tc_maps.ptr, sizeof(maps));
      if (e == cudaSuccess) {
        c->tc_maps.bytes = sizeof(maps);
        e = cudaMemcpy(c->tc_maps.ptr, maps, sizeof(maps), cudaMemcpyHostToDevice);
      }
      if (e != cudaSuccess) {
        fa_kvcache_destroy(c);
        return cuda_fail(e, "cache tensor maps");
      }
    }
  }
  *out = c;
  return FA_OK;
}

int fa_kvcache_destroy(fa_kvcache* cache) {
  if (cache == nullptr) return FA_OK;
  DeviceGuard guard(cache->device);
  if (cache->keys) cudaFree(cache->keys);
  if (cache->values) cudaFree(cache->values);
  cache->work.release();
  cache->staging.release();
  cache->counters.release();
  cache->tc_maps.release();
  cache->proj_work.release();
  cache->proj_counters.release();
  cache->io.release();
  for (cudaEvent_t& e : cache->io_events)
    if (e != nullptr) cudaEventDestroy(e);
  if (cache->copy_stream != nullptr) cudaStreamDestroy(cache->copy_stream);
  if (cache->side_stream != nullptr) cudaStreamDestroy(cache->side_stream);
  delete cache;
  return FA_OK;
}

int fa_kvcache_data(const fa_kvcache* cache, void** keys, void** values, int32_t* shape5,
                    int32_t* dtype) {
  if (int rc = check_cache(cache)) return rc;
  if (keys) *keys = cache->keys;
  if (values) *values = cache->values;
  if (shape5) {
    shape5[0] = cache->layers;
    shape5[1] = cache->heads;
    shape5[2] = cache->kv_heads;
    shape5[3] = cache->head_dim;
    shape5[4] = cache->capacity;
  }
  if (dtype) *dtype = cache->dtype;
  return FA_OK;
}

int fa_kvcache_reserve(fa_kvcache* cache, int32_t rows) {
  if (int rc = check_cache(cache)) return rc;
  if (rows < 1) return fail(FA_ERR_ARG, "rows %d", rows);
  DeviceGuard guard(cache->device);
  const Plan p = plan_span(cache, rows, cache->capacity);
  Work w;
  const size_t staging = size_t(rows) * (cache->heads + 2 * cache->kv_heads) * cache->head_dim * 4 +
                         size_t(rows) * cache->head_dim * 4 + size_t(rows) * cache->heads * cache->head_dim * 4;
  if (int rc = ensure_work(cache, size_t(rows) * cache->heads * cache->head_dim,
                           size_t(rows) * p.chunks * cache->heads, 0, nullptr, &w))
    return rc;
  if (int rc = cache->staging.ensure(staging, nullptr)) return rc;
  // a short span may split a KV head's query heads over several CTAs: a counter per query head
  // covers every split
  if (int rc = ensure_counters(cache, size_t(rows) * cache->heads, nullptr)) return rc;
  FA_CUDA(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  return FA_OK;
}

int fa_kvcache_copy_rows(const fa_kvcache* cache, int32_t rows, void* keys_out,
                         void* values_out, void* stream) {
  if (int rc = check_cache(cache)) return rc;
  if (rows < 0 || rows > cache->capacity)
    return fail(FA_ERR_CAPACITY, "%d rows don't fit a cache of %d", rows, cache->capacity);
  if (keys_out == nullptr || values_out == nullptr) return fail(FA_ERR_ARG, "null output");
  FA_PTR(keys_out, cache->device);
  FA_PTR(values_out, cache->device);
  DeviceGuard guard(cache->device);
  const size_t width = size_t(rows) * cache->head_dim * cache->elem();
  const size_t pitch = size_t(cache->capacity) * cache->head_dim * cache->elem();
  const size_t blocks = size_t(cache->layers) * cache->kv_heads;
  if (width == 0) return FA_OK;
  auto s = static_cast<cudaStream_t>(stream);
  FA_CUDA(cudaMemcpy2DAsync(keys_out, width, cache->keys, pitch, width, blocks,
                            cudaMemcpyDeviceToDevice, s), "copy_rows keys");
  FA_CUDA(cudaMemcpy2DAsync(values_out, width, cache->values, pitch, width, blocks,
                            cudaMemcpyDeviceToDevice, s), "copy_rows values");
  return FA_OK;
}

int fa_kvcache_put_rows(fa_kvcache* cache, int32_t rows, const void* keys, const void* values,
                        void* stream) {
  if (int rc = check_cache(cache)) return rc;
  if (rows < 0 || rows > cache->capacity)
    return fail(FA_ERR_CAPACITY, "%d rows don't fit a cache of %d", rows, cache->capacity);
  if (keys == nullptr || values == nullptr) return fail(FA_ERR_ARG, "null input");
  FA_PTR(keys, cache->device);
  FA_PTR(values, cache->device);
  DeviceGuard guard(cache->device);
  const size_t width = size_t(rows) * cache->head_dim * cache->elem();
  const size_t pitch = size_t(cache->capacity) * cache->head_dim * cache->elem();
  const size_t blocks = size_t(cache->layers) * cache->kv_heads;
  if (width == 0) return FA_OK;
  auto s = static_cast<cudaStream_t>(stream);
  FA_CUDA(cudaMemcpy2DAsync(cache->keys, pitch, keys, width, width, blocks,
                            cudaMemcpyDeviceToDevice, s), "put_rows keys");
  FA_CUDA(cudaMemcpy2DAsync(cache->values, pitch, values, width, width, blocks,
                            cudaMemcpyDeviceToDevice, s), "put_rows values");
  return FA_OK;
}

int fa_rotary_angles(const fa_rotation* rotation, int32_t head_dim, const fa_position* positions,
                     int32_t rows, float* angles_out) {
  if (rotation == nullptr || (rows > 0 && (positions == nullptr || angles_out == nullptr)))
    return fail(FA_ERR_ARG, "null argument");
  if (head_dim < 2 || head_dim % 2 != 0) return fail(FA_ERR_ARG, "head_dim %d", head_dim);
  std::vector<float> inv_freq;
  std::vector<int> axes;
  if (int rc = rotary_frequencies(rotation, head_dim, &inv_freq, &axes)) return rc;
  const int half = head_dim / 2;
  for (int r = 0; r < rows; ++r) {
    const int32_t along[3] = {positions[r].temporal, positions[r].height, positions[r].width};
    float* cos = angles_out + size_t(r) * head_dim;
    float* sin = cos + half;
    for (int i = 0; i < half; ++i) {
      const float angle = float(along[axes[i]]) * inv_freq[i];
      cos[i] = std::cos(angle);
      sin[i] = std::sin(angle);
    }
  }
  return FA_OK;
}

int fa_attention_input(fa_kvcache* cache, int32_t layer, const fa_span* span, int32_t rope,
                       const float* angles, const fa_head_norm* norm, const float* qkv,
                       int64_t qkv_stride, float* q_out, void* stream) {
  if (int rc = check_cache(cache)) return rc;
  if (int rc = check_layer(cache, layer)) return rc;
  std::vector<int> ends;
  if (int rc = check_span(cache, span, &ends)) return rc;
  if (int rc = check_rope(rope, angles)) return rc;
  if (qkv == nullptr && span->rows > 0) return fail(FA_ERR_ARG, "null qkv");
  FA_PTR(qkv, cache->device);
  FA_PTR(angles, cache->device);
  FA_PTR(q_out, cache->device);
  if (qkv_stride < int64_t(cache->heads + 2 * cache->kv_heads) * cache->head_dim)
    return fail(FA_ERR_SHAPE, "qkv rows of %lld values hold fewer than the heads",
                (long long)qkv_stride);
  DeviceGuard guard(cache->device);
  return rope_rows(cache, layer, span, rope, angles, norm, qkv, qkv_stride, q_out,
                   int64_t(cache->heads) * cache->head_dim, 1.0f, true,
                   static_cast<cudaStream_t>(stream));
}

int fa_rotate_queries(int32_t heads, int32_t head_dim, int32_t rows, int32_t rope,
                      const float* angles, const fa_head_norm* norm, const float* qkv,
                      int64_t qkv_stride, float* q_out, int64_t q_out_stride, void* stream) {
  if (heads < 1 || rows < 0) return fail(FA_ERR_ARG, "heads %d rows %d", heads, rows);
  if (!supported_head_dim(head_dim, FA_F32)) return fail(FA_ERR_UNSUPPORTED, "head_dim %d", head_dim);
  if (int rc = check_rope(rope, angles)) return rc;
  if (rows == 0) return FA_OK;
  if (qkv == nullptr || q_out == nullptr) return fail(FA_ERR_ARG, "null qkv or q_out");
  FA_PTR(qkv, current_device());
  FA_PTR(angles, current_device());
  FA_PTR(q_out, current_device());
  if (qkv_stride < int64_t(heads) * head_dim || q_out_stride < int64_t(heads) * head_dim)
    return fail(FA_ERR_SHAPE, "row strides below heads x head_dim");
  fa::RopeArgs a{};
  a.heads = heads;
  a.kv_heads = 1;  // units past the query heads are not visited: keep is off
  a.head_dim = head_dim;
  a.rope = rope;
  a.n_rows = rows;
  a.qkv = qkv;
  a.qkv_stride = qkv_stride;
  a.angles = angles;
  a.q_norm = norm ? norm->q_norm : nullptr;
  a.k_norm = nullptr;
  a.eps = norm ? norm->eps : 0.0f;
  a.q_out = q_out;
  a.q_out_stride = q_out_stride;
  a.q_scale = 1.0f;
  a.keep = 0;
  cudaError_t e = fa::launch_rope(fa::kKtF32, a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rope launch");
  return FA_OK;
}

int fa_attend(fa_kvcache* cache, int32_t layer, const fa_span* span, const float* q,
              int64_t q_stride, float* out, int64_t out_stride, void* stream) {
  if (int rc = check_cache(cache)) return rc;
  if (int rc = check_layer(cache, layer)) return rc;
  std::vector<int> ends;
  if (int rc = check_span(cache, span, &ends)) return rc;
  const int64_t width = int64_t(cache->heads) * cache->head_dim;
  if (span->rows > 0 && (q == nullptr || out == nullptr)) return fail(FA_ERR_ARG, "null q or out");
  FA_PTR(q, cache->device);
  FA_PTR(out, cache->device);
  if (q_stride < width || out_stride < width) return fail(FA_ERR_SHAPE, "row strides below heads x head_dim");
  DeviceGuard guard(cache->device);
  auto s = static_cast<cudaStream_t>(stream);
  if (span->rows == 0) return FA_OK;
  Work w;
  if (span_on_tensor_cores(cache, span) &&
      (cache->dtype == FA_BF16 ||
       ((reinterpret_cast<uintptr_t>(q) % 16) == 0 && (q_stride * 4) % 16 == 0))) {
    if (cache->dtype == FA_F32)
      return attend_rows_tc(cache, layer, span, ends, q, q_stride, out, out_stride, s);
    // bf16 queries for a bf16 cache
    if (int rc = ensure_work(cache, size_t(span->rows) * width, 0, 0, s, &w)) return rc;
    cudaError_t e = fa::launch_prepare_queries(FA_F32, q, q_stride, 0, span->rows, cache->heads,
                                               cache->head_dim, 1.0f, w.q, s, true);
    if (e != cudaSuccess) return cuda_fail(e, "query conversion");
    return attend_rows_tc(cache, layer, span, ends, w.q, width, out, out_stride, s);
  }
  std::vector<fa::Runs> truns;
  if (span_decode_tc(cache, span, ends, &truns)) {
    const DtcPlan plan = plan_decode_tc(cache, truns, span->rows);
    if (int rc = ensure_work(cache, 0, size_t(plan.slots) * cache->heads, 0, s, &w)) return rc;
    std::vector<fa_kvcache*> same(span->rows, cache);
    return attend_batch_tc(same.data(), truns, span->rows, layer, q, q_stride, out, out_stride, s, &w);
  }
  const Plan p = plan_for_span(cache, span, ends);
  if (int rc = ensure_work(cache, 0, size_t(span->rows) * p.chunks * cache->heads, 0, s, &w))
    return rc;
  return attend_rows(cache, layer, span, ends, p, w, q, q_stride, out, out_stride, nullptr, s);
}

int fa_attention(fa_kvcache* cache, int32_t layer, const fa_span* span, int32_t rope,
                 const float* angles, const fa_head_norm* norm, const float* qkv,
                 int64_t qkv_stride, float* out, int64_t out_stride, void* stream) {
  if (int rc = check_cache(cache)) return rc;
  if (int rc = check_layer(cache, layer)) return rc;
  std::vector<int> ends;
  if (int rc = check_span(cache, span, &ends)) return rc;
  if (int rc = check_rope(rope, angles)) return rc;
  const int64_t width = int64_t(cache->heads) * cache->head_dim;
  if (span->rows > 0 && (qkv == nullptr || out == nullptr)) return fail(FA_ERR_ARG, "null qkv or out");
  FA_PTR(qkv, cache->device);
  FA_PTR(angles, cache->device);
  FA_PTR(out, cache->device);
  if (qkv_stride < int64_t(cache->heads + 2 * cache->kv_heads) * cache->head_dim || out_stride < width)
    return fail(FA_ERR_SHAPE, "row strides below the heads' widths");
  if (span->rows == 0) return FA_OK;
  DeviceGuard guard(cache->device);
  auto s = static_cast<cudaStream_t>(stream);
  Work w;
  if (span_on_tensor_cores(cache, span)) {
    // rotated queries in the cache's element type, for the TMA loads of the tensor-core kernel
    if (int rc = ensure_work(cache, size_t(span->rows) * width, 0, 0, s, &w)) return rc;
    if (int rc = rope_rows(cache, layer, span, rope, angles, norm, qkv, qkv_stride, w.q, width,
                           1.0f, true, s, cache->dtype == FA_BF16))
      return rc;
    return attend_rows_tc(cache, layer, span, ends, w.q, width, out, out_stride, s);
  }
  std::vector<fa::Runs> truns;
  if (span_decode_tc(cache, span, ends, &truns)) {
    const DtcPlan plan = plan_decode_tc(cache, truns, span->rows);
    if (int rc = ensure_work(cache, size_t(span->rows) * width, size_t(plan.slots) * cache->heads,
                             0, s, &w))
      return rc;
    if (int rc = rope_rows(cache, layer, span, rope, angles, norm, qkv, qkv_stride, w.q, width,
                           1.0f, true, s))
      return rc;
    std::vector<fa_kvcache*> same(span->rows, cache);
    return attend_batch_tc(same.data(), truns, span->rows, layer, w.q, width, out, out_stride, s,
                           &w);
  }
  const Plan p = plan_for_span(cache, span, ends);
  if (int rc = ensure_work(cache, size_t(span->rows) * width,
                           size_t(span->rows) * p.chunks * cache->heads, 0, s, &w))
    return rc;
  if (int rc = rope_rows(cache, layer, span, rope, angles, norm, qkv, qkv_stride, w.q, width,
                         1.0f, true, s))
    return rc;
  return attend_rows(cache, layer, span, ends, p, w, w.q, width, out, out_stride, nullptr, s);
}

int fa_attention_host(fa_kvcache* cache, int32_t layer, const fa_span* span, int32_t rope,
                      const float* angles_host, const fa_head_norm* norm, const float* qkv_host,
                      int64_t qkv_stride, float* out_host, int64_t out_stride, void* stream) {
  if (int rc = check_cache(cache)) return rc;
  if (span == nullptr) return fail(FA_ERR_ARG, "null span");
  if (span->rows == 0) return FA_OK;
  if (qkv_host == nullptr || out_host == nullptr) return fail(FA_ERR_ARG, "null qkv or out");
  if (int rc = check_rope(rope, angles_host)) return rc;
  if (qkv_stride < int64_t(cache->heads + 2 * cache->kv_heads) * cache->head_dim ||
      out_stride < int64_t(cache->heads) * cache->head_dim)
    return fail(FA_ERR_SHAPE, "row strides below the heads' widths");
  DeviceGuard guard(cache->device);
  auto s = static_cast<cudaStream_t>(stream);
  const int rows = span->rows;
  const int64_t width = int64_t(cache->heads) * cache->head_dim;
  const int64_t units = int64_t(cache->heads + 2 * cache->kv_heads) * cache->head_dim;
  // Staging: the rows' qkv (packed to the units' width), their angles and outputs.
  const size_t staging = size_t(rows) * units * 4 + size_t(rows) * cache->head_dim * 4 +
                         size_t(rows) * width * 4;
  if (int rc = cache->staging.ensure(staging, s)) return rc;
  float* qkv_dev = static_cast<float*>(cache->staging.ptr);
  float* angles_dev = qkv_dev + size_t(rows) * units;
  float* out_dev = angles_dev + size_t(rows) * cache->head_dim;
  FA_CUDA(rows_to_device(qkv_dev, units, qkv_host, qkv_stride, rows, s), "qkv to device");
  if (rope != FA_ROPE_NONE)
    FA_CUDA(cudaMemcpyAsync(angles_dev, angles_host, size_t(rows) * cache->head_dim * 4,
                            cudaMemcpyHostToDevice, s), "angles to device");
  if (int rc = fa_attention(cache, layer, span, rope, rope != FA_ROPE_NONE ? angles_dev : nullptr,
                            norm, qkv_dev, units, out_dev, width, stream))
    return rc;
  FA_CUDA(cudaMemcpy2DAsync(out_host, out_stride * 4, out_dev, width * 4, width * 4, rows,
                            cudaMemcpyDeviceToHost, s), "out to host");
  FA_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
  return FA_OK;
}

namespace {

// The checks and the per-row key runs of a batch of one-row spans over caches of one shape.
int check_batch(fa_kvcache* const* caches, const fa_span* spans, int32_t batch, int32_t layer,
                std::vector<fa::Runs>* runs, int64_t* total_keys) {
  if (caches == nullptr || spans == nullptr) return fail(FA_ERR_ARG, "null caches or spans");
  if (batch < 0 || batch > 1024) return fail(FA_ERR_ARG, "batch %d (1..1024)", batch);
  if (batch == 0) return FA_OK;
  const fa_kvcache* c0 = caches[0];
  if (int rc = check_cache(c0)) return rc;
  if (int rc = check_layer(c0, layer)) return rc;
  runs->assign(batch, fa::Runs{0, 0, 0, 0});
  std::vector<int> ends;
  *total_keys = 0;
  for (int i = 0; i < batch; ++i) {
    const fa_kvcache* c = caches[i];
    if (int rc = check_cache(c)) return rc;
    if (c->heads != c0->heads || c->kv_heads != c0->kv_heads || c->head_dim != c0->head_dim ||
        c->layers != c0->layers || c->dtype != c0->dtype || c->device != c0->device)
      return fail(FA_ERR_SHAPE, "sequence %d's cache differs in shape from the first", i);
    if (spans[i].rows != 1) return fail(FA_ERR_ARG, "batched spans are one row (decode)");
    if (int rc = check_span(c, &spans[i], &ends)) return rc;
    // Mask::keys of the row: under Groups the state's run and the row's own group (two runs,
    // which decode on the CUDA cores)
    (*runs)[i] = fa::mask_runs(spans[i].mask.kind, spans[i].mask.window, spans[i].mask.state,
                               int(ends.size()), ends.data(), spans[i].first, spans[i].first + 1);
    *total_keys += (*runs)[i].n0 + (*runs)[i].n1;
  }
  return FA_OK;
}

// The chunk length, in tiles, of a batch decode on the split-KV kernel: the one of least
// modelled time among 16..64 tiles. The CTAs run in waves of the SMs' resident slots, the units
// of a length spread evenly over them. A wave is bound both by its bytes at the HBM rate (a) and
// by its longest chunk at one CTA's own streaming rate, two stages of K and V in flight (b); the
// two overlap only in part, so a wave takes cbrt(a^3 + b^3), plus 2 us. Fitted on B200 to a
// GPU's share of C3 at 1, 2, 4 and 8 GPUs (64, 32, 16 and 8 sequences, f32, head_dim 128;
// lengths of 8..64 tiles): 6.9 TB/s, 32.8 GB/s per CTA (one 32 KB tile a microsecond). Against
// eight lengths timed in interleaved rounds on one GPU, its choice (63, 46, 47 and 22 tiles) runs
// within 2 % of the fastest at every size; the fixed floor of 32 tiles it replaces left 16
// sequences in 1.37 waves (114 us against 95 us), and lengths whose last wave is barely begun
// (1.05, 1.14 and 2.25 waves) are the slowest. Below 16 tiles the CTAs' fixed costs dominate
// (9 tiles: 367 us for 64 sequences, against 340-346 us for 22-63).
int batch_chunk_tiles(const fa_kvcache* c0, const Plan& base, const std::vector<fa::Runs>& runs,
                      int batch, int tile, int kt) {
  constexpr int kMinTiles = 16, kMaxTiles = 64;
  constexpr double kHbmTilesPerUs = 210.0;  // the whole GPU, reading (32 KB tiles)
  constexpr double kCtaTilesPerUs = 1.0;    // one CTA
  constexpr double kWaveUs = 2.0;
  fa::AttendLaunch probe{kt, base.g, true, nullptr, nullptr, 0};
  const int resident = attend_resident_d(c0->head_dim, probe);
  const int64_t slots = int64_t(std::max(c0->dev->sms, 1)) * std::max(resident, 1);
  // Each row in tiles, at least one: its chunks of t tiles are ceil(tiles / t) (= ceil(keys /
  // (t x tile))), in 32-bit arithmetic (a row holds fewer than 2^31 keys). This search runs on
  // the host before every batch launch: 16 rows x 49 lengths took 7.5 us in 64-bit divisions.
  int64_t longest = 1, keys_total = 0;
  std::vector<uint32_t> row_tiles(batch);
  for (int i = 0; i < batch; ++i) {
    const int64_t n = runs[i].n0 + runs[i].n1;
    longest = std::max(longest, n);
    keys_total += n;
    row_tiles[i] = uint32_t(std::max<int64_t>(1, (n + tile - 1) / tile));
  }
  const double tiles_total = double(keys_total) * base.kv_groups / tile;
  const int top = int(std::min<int64_t>(kMaxTiles, std::max<int64_t>(kMinTiles, (longest + tile - 1) / tile)));
  int best = top;
  double best_us = 1e300;
  for (int t = top; t >= kMinTiles; --t) {  // ties go to the longer chunk: fewer partials
    const uint32_t ut = uint32_t(t);
    int64_t units = 0;
    for (int i = 0; i < batch; ++i) units += (row_tiles[i] + ut - 1) / ut;
    units *= base.kv_groups;
    const double per_unit = tiles_total / double(units);
    const double bt = t / kCtaTilesPerUs, b3 = bt * bt * bt;
    auto wave = [&](int64_t n) {
      const double a = n * per_unit / kHbmTilesPerUs;
      return std::cbrt(a * a * a + b3) + kWaveUs;
    };
    const int64_t full = units / slots, rest = units % slots;
    const double us = double(full) * wave(slots) + (rest > 0 ? wave(rest) : 0.0);
    if (us < best_us * (1.0 - 1e-9)) {
      best_us = us;
      best = t;
    }
  }
  return best;
}

}  // namespace

namespace {

// The fused projection's launch plan (fa_project.cu): rows per pass, rows per CTA (at most 16),
// and the split of the hidden dimension into chunks of whole 128-value steps (at most 1024) that
// gives about four waves' worth of CTAs (several resident per SM: the weights stream with more
// loads in flight). Measured on B200 with a 6144 x 4096 projection: for one row, four waves ran
// 1.2x as fast as two (31 vs 37 us per graph replay, L2 flushed); for 16 and 64 rows, 16-row
// blocks and 1024-value chunks ran 1.7x as fast as 64-row blocks with the whole chunk of every
// row staged in one CTA's shared memory.
struct ProjectPlan {
  int nr, row_block, row_blocks, splits, chunk;
  size_t smem;
};

constexpr int kProjectSmemFloats = 200 * 1024 / 4;

ProjectPlan plan_project(int rows, int hidden, int units, int head_dim, int sms) {
  ProjectPlan p{};
  p.nr = rows == 1 ? 1 : (rows <= 4 ? 4 : 8);
  p.row_block = std::min((rows + p.nr - 1) / p.nr * p.nr, 16);
  p.row_blocks = (rows + p.row_block - 1) / p.row_block;
  const int steps = (hidden + 127) / 128;
  const int64_t blocks = int64_t(units) * p.row_blocks;
  const int64_t want = std::max<int64_t>((4 * int64_t(std::max(sms, 1)) + blocks - 1) / blocks, 1);
  const int splits = int(std::min<int64_t>(want, steps));
  const int max_chunk =
      std::max((kProjectSmemFloats - p.row_block * head_dim) / p.row_block / 128 * 128, 128);
  p.chunk = std::min(std::min((steps + splits - 1) / splits * 128, max_chunk), 1024);
  p.splits = (hidden + p.chunk - 1) / p.chunk;
  p.smem = size_t(p.row_block) * (p.chunk + head_dim) * sizeof(float);
  return p;
}

int check_linear(const fa_kvcache* c, const fa_linear* lin, const float* x, int64_t x_stride) {
  if (lin == nullptr || lin->weight == nullptr) return fail(FA_ERR_ARG, "null qkv weights");
  if (x == nullptr) return fail(FA_ERR_ARG, "null input rows");
  const int outputs = (c->heads + 2 * c->kv_heads) * c->head_dim;
  if (lin->outputs != outputs)
    return fail(FA_ERR_SHAPE, "the qkv projection gives %d outputs, the heads need %d",
                lin->outputs, outputs);
  if (lin->inputs < 1 || lin->weight_stride < lin->inputs || x_stride < lin->inputs)
    return fail(FA_ERR_SHAPE, "inputs %d, weight stride %lld, input stride %lld", lin->inputs,
                (long long)lin->weight_stride, (long long)x_stride);
  if (c->head_dim % 8 != 0)
    return fail(FA_ERR_UNSUPPORTED, "the fused projection takes head_dim a multiple of 8");
  if (lin->inputs % 4 || lin->weight_stride % 4 || x_stride % 4 ||
      reinterpret_cast<uintptr_t>(lin->weight) % 16 || reinterpret_cast<uintptr_t>(x) % 16)
    return fail(FA_ERR_UNSUPPORTED, "weight and input rows must start on 16-byte boundaries");
  FA_PTR(lin->weight, c->device);
  FA_PTR(lin->bias, c->device);
  FA_PTR(x, c->device);
  return FA_OK;
}

// From this many rows the projection runs on the tensor cores (fa_project_tc.cu) and then the
// RoPE + keep kernel; below it, in the fused CUDA-core kernel, bound by the weight bytes.
constexpr int kProjectTcRows = 16;

// Splits of the hidden dimension for the tensor-core projection: enough CTAs (one an SM, each
// holding about 200 KB of shared memory) to fill the SMs once, at most 8, with at least 4
// k-blocks each.
int project_tc_splits(int64_t blocks, int k_blocks, int sms) {
  int64_t s = std::max<int64_t>(1, sms / std::max<int64_t>(blocks, 1));
  s = std::min<int64_t>(s, 8);
  s = std::min<int64_t>(s, std::max(1, k_blocks / 4));
  return int(s);
}

// The tensor-core projection of `rows` rows into qkv_out (or c0's projection workspace), then the
// RoPE + keep kernel over them.
int launch_projection_tc(fa_kvcache* c0, const fa_linear* lin, const float* x, int64_t x_stride,
                         int rows, const fa::RopeArgs& ra, float* qkv_out, int64_t qkv_out_stride,
                         cudaStream_t s) {
  fa::ProjectTcArgs t{};
  t.x = x;
  t.x_stride = x_stride;
  t.weight = lin->weight;
  t.w_stride = lin->weight_stride;
  t.bias = lin->bias;
  t.hidden = lin->inputs;
  t.outputs = lin->outputs;
  t.rows = rows;
  t.k_blocks = (lin->inputs + 31) / 32;
  t.qkv = qkv_out;
  t.qkv_stride = qkv_out_stride;
  t.err = c0->dev->err;
  const int bn = fa::project_tc_rows_per_tile(rows);
  const int64_t tiles = int64_t((lin->outputs + 127) / 128) * ((rows + bn - 1) / bn);
  t.splits = project_tc_splits(tiles, t.k_blocks, c0->dev->sms);
  // the workspace: the projected rows (when the caller keeps none), then the splits' partials
  const size_t qkv_bytes = qkv_out ? 0 : align_up(size_t(rows) * lin->outputs * sizeof(float), 256);
  const size_t part_bytes = t.splits > 1 ? size_t(tiles) * t.splits * bn * 128 * sizeof(float) : 0;
  if (qkv_bytes + part_bytes > 0) {
    if (int rc = c0->proj_work.ensure(qkv_bytes + part_bytes, s)) return rc;
    unsigned char* w = static_cast<unsigned char*>(c0->proj_work.ptr);
    if (qkv_out == nullptr) {
      t.qkv = reinterpret_cast<float*>(w);
      t.qkv_stride = lin->outputs;
    }
    t.partials = reinterpret_cast<float*>(w + qkv_bytes);
  }
  if (t.splits > 1) {
    const int epoch = c0->dev->epoch.load();
    if (size_t(tiles) * sizeof(int) > c0->proj_counters.bytes || c0->proj_epoch != epoch) {
      if (int rc = c0->proj_counters.ensure(size_t(tiles) * sizeof(int), s)) return rc;
      FA_CUDA(cudaMemsetAsync(c0->proj_counters.ptr, 0, c0->proj_counters.bytes, s),
              "clear projection counters");
      c0->proj_epoch = epoch;
    }
    t.counters = static_cast<int*>(c0->proj_counters.ptr);
  }
  cudaError_t e = fa::launch_project_tc(t, s);
  if (e != cudaSuccess) return cuda_fail(e, "tensor-core projection launch");
  fa::RopeArgs r = ra;
  r.qkv = t.qkv;
  r.qkv_stride = t.qkv_stride;
  e = fa::launch_rope(c0->dtype == FA_F32 ? fa::kKtF32 : fa::kKtBf16, r, s);
  if (e != cudaSuccess) return cuda_fail(e, "rope launch");
  return FA_OK;
}

// One launch of the fused projection over `rows` rows: the RopeArgs say where each row's keys and
// values go; the partials and counters live in c0's projection workspace.
int launch_projection(fa_kvcache* c0, const fa_linear* lin, const float* x, int64_t x_stride,
                      int rows, const fa::RopeArgs& ra, float* qkv_out, int64_t qkv_out_stride,
                      cudaStream_t s) {
  if (rows == 0) return FA_OK;
  if (rows >= kProjectTcRows)
    return launch_projection_tc(c0, lin, x, x_stride, rows, ra, qkv_out, qkv_out_stride, s);
  const int units = c0->heads + 2 * c0->kv_heads;
  const ProjectPlan plan = plan_project(rows, lin->inputs, units, c0->head_dim, c0->dev->sms);
  fa::ProjectArgs p{};
  p.x = x;
  p.x_stride = x_stride;
  p.weight = lin->weight;
  p.w_stride = lin->weight_stride;
  p.bias = lin->bias;
  p.hidden = lin->inputs;
  p.rows = rows;
  p.row_block = plan.row_block;
  p.splits = plan.splits;
  p.chunk = plan.chunk;
  p.qkv_out = qkv_out;
  p.qkv_out_stride = qkv_out_stride;
  if (plan.splits > 1) {
    const size_t blocks = size_t(units) * plan.row_blocks;
    if (int rc = c0->proj_work.ensure(blocks * plan.splits * plan.row_block * c0->head_dim * 4, s))
      return rc;
    const int epoch = c0->dev->epoch.load();
    if (blocks * sizeof(int) > c0->proj_counters.bytes || c0->proj_epoch != epoch) {
      if (int rc = c0->proj_counters.ensure(blocks * sizeof(int), s)) return rc;
      FA_CUDA(cudaMemsetAsync(c0->proj_counters.ptr, 0, c0->proj_counters.bytes, s),
              "clear projection counters");
      c0->proj_epoch = epoch;
    }
    p.partials = static_cast<float*>(c0->proj_work.ptr);
    p.counters = static_cast<int*>(c0->proj_counters.ptr);
  }
  cudaError_t e = fa::launch_project(c0->dtype == FA_F32 ? fa::kKtF32 : fa::kKtBf16, plan.nr, p,
                                     ra, plan.smem, s);
  if (e != cudaSuccess) return cuda_fail(e, "projection launch");
  return FA_OK;
}

}  // namespace

int fa_attention_input_projected(fa_kvcache* cache, int32_t layer, const fa_span* span,
                                 int32_t rope, const float* angles, const fa_head_norm* norm,
                                 const fa_linear* qkv, const float* x, int64_t x_stride,
                                 float* q_out, float* qkv_out, int64_t qkv_out_stride,
                                 void* stream) {
  if (int rc = check_cache(cache)) return rc;
  if (int rc = check_layer(cache, layer)) return rc;
  std::vector<int> ends;
  if (int rc = check_span(cache, span, &ends)) return rc;
  if (int rc = check_rope(rope, angles)) return rc;
  if (span->rows == 0) return FA_OK;
  if (int rc = check_linear(cache, qkv, x, x_stride)) return rc;
  FA_PTR(angles, cache->device);
  FA_PTR(q_out, cache->device);
  FA_PTR(qkv_out, cache->device);
  if (qkv_out != nullptr && qkv_out_stride < qkv->outputs)
    return fail(FA_ERR_SHAPE, "qkv_out rows narrower than the projection");
  DeviceGuard guard(cache->device);
  fa::RopeArgs a{};
  a.heads = cache->heads;
  a.kv_heads = cache->kv_heads;
  a.head_dim = cache->head_dim;
  a.rope = rope;
  a.n_rows = span->rows;
  a.angles = angles;
  a.q_norm = norm ? norm->q_norm : nullptr;
  a.k_norm = norm ? norm->k_norm : nullptr;
  a.eps = norm ? norm->eps : 0.0f;
  a.q_out = q_out;
  a.q_out_stride = int64_t(cache->heads) * cache->head_dim;
  a.q_scale = 1.0f;
  a.keep = 1;
  a.batch = 0;
  a.first = span->first;
  a.keep_rows[0].k = const_cast<unsigned char*>(layer_ptr(cache, cache->keys, layer));
  a.keep_rows[0].v = const_cast<unsigned char*>(layer_ptr(cache, cache->values, layer));
  a.keep_rows[0].capacity = cache->capacity;
  return launch_projection(cache, qkv, x, x_stride, span->rows, a, qkv_out, qkv_out_stride,
                           static_cast<cudaStream_t>(stream));
}

int fa_attention_input_projected_batch(fa_kvcache* const* caches, const fa_span* spans,
                                       int32_t batch, int32_t layer, int32_t rope,
                                       const float* angles, const fa_head_norm* norm,
                                       const fa_linear* qkv, const float* x, int64_t x_stride,
                                       float* q_out, int64_t q_out_stride, void* stream) {
  std::vector<fa::Runs> runs;
  int64_t total_keys = 0;
  if (int rc = check_batch(caches, spans, batch, layer, &runs, &total_keys)) return rc;
  if (batch == 0) return FA_OK;
  if (int rc = check_rope(rope, angles)) return rc;
  fa_kvcache* c0 = caches[0];
  if (int rc = check_linear(c0, qkv, x, x_stride)) return rc;
  FA_PTR(angles, c0->device);
  FA_PTR(q_out, c0->device);
  if (q_out != nullptr && q_out_stride < int64_t(c0->heads) * c0->head_dim)
    return fail(FA_ERR_SHAPE, "q_out rows narrower than the query heads");
  DeviceGuard guard(c0->device);
  auto s = static_cast<cudaStream_t>(stream);
  for (int first = 0; first < batch; first += fa::kMaxBatchRows) {
    const int n = std::min(batch - first, fa::kMaxBatchRows);
    fa::RopeArgs ra{};
    ra.heads = c0->heads;
    ra.kv_heads = c0->kv_heads;
    ra.head_dim = c0->head_dim;
    ra.rope = rope;
    ra.n_rows = n;
    ra.angles = angles ? angles + int64_t(first) * c0->head_dim : nullptr;
    ra.q_norm = norm ? norm->q_norm : nullptr;
    ra.k_norm = norm ? norm->k_norm : nullptr;
    ra.eps = norm ? norm->eps : 0.0f;
    ra.q_out = q_out ? q_out + int64_t(first) * q_out_stride : nullptr;
    ra.q_out_stride = q_out_stride;
    ra.q_scale = 1.0f;
    ra.keep = 1;
    ra.batch = 1;
    for (int i = 0; i < n; ++i) {
      const fa_kvcache* c = caches[first + i];
      ra.keep_rows[i].k = const_cast<unsigned char*>(layer_ptr(c, c->keys, layer));
      ra.keep_rows[i].v = const_cast<unsigned char*>(layer_ptr(c, c->values, layer));
      ra.keep_rows[i].capacity = c->capacity;
      ra.keep_rows[i].position = spans[first + i].first;
    }
    if (int rc = launch_projection(c0, qkv, x + int64_t(first) * x_stride, x_stride, n, ra,
                                   nullptr, 0, s))
      return rc;
  }
  return FA_OK;
}

int fa_attention_input_batch(fa_kvcache* const* caches, const fa_span* spans, int32_t batch,
                             int32_t layer, int32_t rope, const float* angles,
                             const fa_head_norm* norm, const float* qkv, int64_t qkv_stride,
                             float* q_out, int64_t q_out_stride, void* stream) {
  std::vector<fa::Runs> runs;
  int64_t total_keys = 0;
  if (int rc = check_batch(caches, spans, batch, layer, &runs, &total_keys)) return rc;
  if (batch == 0) return FA_OK;
  if (int rc = check_rope(rope, angles)) return rc;
  fa_kvcache* c0 = caches[0];
  const int64_t width = int64_t(c0->heads) * c0->head_dim;
  if (qkv == nullptr) return fail(FA_ERR_ARG, "null qkv");
  FA_PTR(qkv, c0->device);
  FA_PTR(angles, c0->device);
  FA_PTR(q_out, c0->device);
  if (qkv_stride < int64_t(c0->heads + 2 * c0->kv_heads) * c0->head_dim ||
      (q_out != nullptr && q_out_stride < width))
    return fail(FA_ERR_SHAPE, "row strides below the heads' widths");
  DeviceGuard guard(c0->device);
  auto s = static_cast<cudaStream_t>(stream);
  const int kt = c0->dtype == FA_F32 ? fa::kKtF32 : fa::kKtBf16;
  for (int first = 0; first < batch; first += fa::kMaxBatchRows) {
    const int n = std::min(batch - first, fa::kMaxBatchRows);
    fa::RopeArgs ra{};
    ra.heads = c0->heads;
    ra.kv_heads = c0->kv_heads;
    ra.head_dim = c0->head_dim;
    ra.rope = rope;
    ra.n_rows = n;
    ra.qkv = qkv + int64_t(first) * qkv_stride;
    ra.qkv_stride = qkv_stride;
    ra.angles = angles ? angles + int64_t(first) * c0->head_dim : nullptr;
    ra.q_norm = norm ? norm->q_norm : nullptr;
    ra.k_norm = norm ? norm->k_norm : nullptr;
    ra.eps = norm ? norm->eps : 0.0f;
    ra.q_out = q_out ? q_out + int64_t(first) * q_out_stride : nullptr;
    ra.q_out_stride = q_out_stride;
    ra.q_scale = 1.0f;
    ra.keep = 1;
    ra.batch = 1;
    for (int i = 0; i < n; ++i) {
      const fa_kvcache* c = caches[first + i];
      ra.keep_rows[i].k = const_cast<unsigned char*>(layer_ptr(c, c->keys, layer));
      ra.keep_rows[i].v = const_cast<unsigned char*>(layer_ptr(c, c->values, layer));
      ra.keep_rows[i].capacity = c->capacity;
      ra.keep_rows[i].position = spans[first + i].first;
    }
    cudaError_t e = fa::launch_rope(kt, ra, s);
    if (e != cudaSuccess) return cuda_fail(e, "rope launch");
  }
  return FA_OK;
}

int fa_attend_batch(fa_kvcache* const* caches, const fa_span* spans, int32_t batch,
                    int32_t layer, const float* q, int64_t q_stride, float* out,
                    int64_t out_stride, void* stream) {
  std::vector<fa::Runs> runs;
  int64_t total_keys = 0;
  if (int rc = check_batch(caches, spans, batch, layer, &runs, &total_keys)) return rc;
  if (batch == 0) return FA_OK;
  fa_kvcache* c0 = caches[0];
  const int64_t width = int64_t(c0->heads) * c0->head_dim;
  if (q == nullptr || out == nullptr) return fail(FA_ERR_ARG, "null q or out");
  FA_PTR(q, c0->device);
  FA_PTR(out, c0->device);
  if (q_stride < width || out_stride < width) return fail(FA_ERR_SHAPE, "row strides below heads x head_dim");
  DeviceGuard guard(c0->device);
  auto s = static_cast<cudaStream_t>(stream);
  if (decode_on_tensor_cores(caches, runs, batch))
    return attend_batch_tc(caches, runs, batch, layer, q, q_stride, out, out_stride, s);
  const Plan base = plan_span(c0, 1, 1, false);
  const int kt = c0->dtype == FA_F32 ? fa::kKtF32 : fa::kKtBf16;
  const int tile = fa::tile_keys(kernel_dim(c0->head_dim), kt);
  const int64_t chunk_keys = int64_t(tile) * batch_chunk_tiles(c0, base, runs, batch, tile, kt);
  // Chunks and partial slots of every row, then one launch per kMaxBatchRows rows.
  std::vector<int> chunks(batch), part_base(batch);
  int64_t slots = 0;
  for (int i = 0; i < batch; ++i) {
    const int64_t n = runs[i].n0 + runs[i].n1;
    chunks[i] = int(std::max<int64_t>(1, (n + chunk_keys - 1) / chunk_keys));
    part_base[i] = int(slots);
    slots += chunks[i];
  }
  Work w;
  if (int rc = ensure_work(c0, 0, size_t(slots) * c0->heads, 0, s, &w)) return rc;
  if (int rc = ensure_counters(c0, size_t(batch) * base.kv_groups, s)) return rc;
  for (int first = 0; first < batch; first += fa::kMaxBatchRows) {
    const int n = std::min(batch - first, fa::kMaxBatchRows);
    fa::BatchArgs ba{};
    fill_common(&ba.c, c0, base);
    ba.c.q = q + int64_t(first) * q_stride;
    ba.c.q_stride = q_stride;
    ba.c.out = out + int64_t(first) * out_stride;
    ba.c.out_stride = out_stride;
    ba.c.partial_out = nullptr;
    ba.c.part_o = w.part_o;
    ba.c.part_ml = w.part_ml;
    ba.c.counters = static_cast<int*>(c0->counters.ptr) + int64_t(first) * base.kv_groups;
    ba.n = n;
    int units = 0;
    for (int i = 0; i < n; ++i) {
      const fa_kvcache* c = caches[first + i];
      fa::BatchRow& br = ba.rows[i];
      br.k = layer_ptr(c, c->keys, layer);
      br.v = layer_ptr(c, c->values, layer);
      br.capacity = c->capacity;
      br.runs = runs[first + i];
      br.chunks = chunks[first + i];
      br.unit_begin = units;
      br.part_base = part_base[first + i];
      units += base.kv_groups * br.chunks;
    }
    fa::AttendLaunch l{kt, base.g, true, nullptr, &ba, units};
    cudaError_t e = launch_attend_d(c0->head_dim, l, s);
    if (e != cudaSuccess) return cuda_fail(e, "attend launch");
  }
  return FA_OK;
}

int fa_attention_batch(fa_kvcache* const* caches, const fa_span* spans, int32_t batch,
                       int32_t layer, int32_t rope, const float* angles,
                       const fa_head_norm* norm, const float* qkv, int64_t qkv_stride,
                       float* out, int64_t out_stride, void* stream) {
  std::vector<fa::Runs> runs;
  int64_t total_keys = 0;
  if (int rc = check_batch(caches, spans, batch, layer, &runs, &total_keys)) return rc;
  if (batch == 0) return FA_OK;
  fa_kvcache* c0 = caches[0];
  const int64_t width = int64_t(c0->heads) * c0->head_dim;
  DeviceGuard guard(c0->device);
  auto s = static_cast<cudaStream_t>(stream);
  // The rotated queries go to the first cache's staging buffer (its workspace holds partials).
  if (int rc = c0->staging.ensure(size_t(batch) * width * 4, s)) return rc;
  float* q = static_cast<float*>(c0->staging.ptr);
  if (int rc = fa_attention_input_batch(caches, spans, batch, layer, rope, angles, norm, qkv,
                                        qkv_stride, q, width, stream))
    return rc;
  return fa_attend_batch(caches, spans, batch, layer, q, width, out, out_stride, stream);
}

int fa_attention_batch_host(fa_kvcache* const* caches, const fa_span* spans, int32_t batch,
                            int32_t layer, int32_t rope, const float* angles_host,
                            const fa_head_norm* norm, const float* qkv_host, int64_t qkv_stride,
                            float* out_host, int64_t out_stride, void* stream) {
  std::vector<fa::Runs> runs;
  int64_t total_keys = 0;
  if (int rc = check_batch(caches, spans, batch, layer, &runs, &total_keys)) return rc;
  if (batch == 0) return FA_OK;
  if (qkv_host == nullptr || out_host == nullptr) return fail(FA_ERR_ARG, "null qkv or out");
  if (int rc = check_rope(rope, angles_host)) return rc;
  fa_kvcache* c0 = caches[0];
  const int d = c0->head_dim;
  const int64_t width = int64_t(c0->heads) * d;
  const int64_t units = int64_t(c0->heads + 2 * c0->kv_heads) * d;
  if (qkv_stride < units || out_stride < width)
    return fail(FA_ERR_SHAPE, "row strides below the heads' widths");
  DeviceGuard guard(c0->device);
  auto s = static_cast<cudaStream_t>(stream);
  // Staging on the first cache: the rows' qkv (packed to the units' width), angles and outputs.
  const size_t staging = size_t(batch) * (units + d + width) * 4;
  if (int rc = c0->io.ensure(staging, s)) return rc;
  float* qkv_dev = static_cast<float*>(c0->io.ptr);
  float* angles_dev = qkv_dev + size_t(batch) * units;
  // A pinned output that this device can address (mapped host memory) takes the attention
  // kernels' stores directly, each row over PCIe as it is merged, during the kernel: no copy of
  // the outputs after the last group. Pageable output goes through device staging and a copy.
  float* out_dev = angles_dev + size_t(batch) * d;
  int64_t out_dev_stride = width;
  bool out_mapped = false;
  {
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, out_host) != cudaSuccess) {
      cudaGetLastError();
    } else if (attr.type == cudaMemoryTypeHost && attr.devicePointer != nullptr) {
      out_dev = static_cast<float*>(attr.devicePointer);
      out_dev_stride = out_stride;
      out_mapped = true;
    }
  }
  // Two groups of consecutive sequences once the batch is large enough for each group's launch
  // to fill the SMs (each group's keys are chunked over the whole GPU): the first a quarter of
  // the keys, so that its rows (a quarter of the copy) land soon and the GPU starts on them while
  // the others' rows arrive; the second group runs on a second stream, concurrent with the
  // first, so that its launch fills the SMs the first one's last wave leaves idle. Measured on
  // B200 with C3's 64 sequences (pinned memory, mean per step, f32 / bf16 caches): the groups
  // one after the other on the caller's stream 0.422 / 0.291 ms; concurrent, halves of the keys
  // 0.403-0.407 / 0.257-0.279, a quarter first 0.402 / 0.254 (an eighth 0.405-0.416; four
  // concurrent quarters 0.402 / 0.317).
  const int groups = batch >= 16 ? 2 : 1;
  if (groups == 1) {
    FA_CUDA(rows_to_device(qkv_dev, units, qkv_host, qkv_stride, batch, s), "qkv to device");
    if (rope != FA_ROPE_NONE)
      FA_CUDA(cudaMemcpyAsync(angles_dev, angles_host, size_t(batch) * d * 4,
                              cudaMemcpyHostToDevice, s), "angles to device");
    if (int rc = fa_attention_batch(caches, spans, batch, layer, rope,
                                    rope != FA_ROPE_NONE ? angles_dev : nullptr, norm, qkv_dev,
                                    units, out_dev, out_dev_stride, stream))
      return rc;
    if (!out_mapped)
      FA_CUDA(cudaMemcpy2DAsync(out_host, out_stride * 4, out_dev, width * 4, width * 4, batch,
                                cudaMemcpyDeviceToHost, s), "out to host");
    FA_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    return FA_OK;
  }
  static_assert(kMaxHostGroups == 2, "groups");
  if (c0->copy_stream == nullptr)
    FA_CUDA(cudaStreamCreateWithFlags(&c0->copy_stream, cudaStreamNonBlocking), "copy stream");
  if (c0->side_stream == nullptr)
    FA_CUDA(cudaStreamCreateWithFlags(&c0->side_stream, cudaStreamNonBlocking), "side stream");
  for (cudaEvent_t& e : c0->io_events)
    if (e == nullptr) FA_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "copy event");
  cudaStream_t cs = c0->copy_stream;
  cudaEvent_t* in_ready = c0->io_events;
  cudaEvent_t* done = c0->io_events + kMaxHostGroups;
  cudaEvent_t side_end = c0->io_events[2 * kMaxHostGroups];
  int bounds[3] = {0, batch, batch};
  {
    int64_t seen = 0;
    for (int i = 0; i + 1 < batch; ++i) {
      seen += runs[i].n0 + runs[i].n1;
      if (seen * 4 >= total_keys) {
        bounds[1] = i + 1;
        break;
      }
    }
  }
  // A group's launches use its first cache's workspace, queries and counters: the groups run
  // concurrently only when those caches are distinct (a batch may name a cache twice).
  const bool concurrent = bounds[1] == batch || caches[0] != caches[bounds[1]];
  cudaStream_t side = concurrent ? c0->side_stream : s;
  // The copy stream and the side stream start after the caller's earlier work; the copy stream
  // takes each group's rows in, then (unmapped output) each group's outputs out once that group
  // has attended. The host issues a group's copy and then its launches before the next group's
  // copy: the first group's launches are the host's share of the call's critical path.
  FA_CUDA(cudaEventRecord(done[0], s), "copy event");
  FA_CUDA(cudaStreamWaitEvent(cs, done[0], 0), "copy stream wait");
  if (side != s) FA_CUDA(cudaStreamWaitEvent(side, done[0], 0), "side stream wait");
  int rc = FA_OK;
  for (int g = 0; g < groups && rc == FA_OK; ++g) {
    const int b0 = bounds[g], n = bounds[g + 1] - bounds[g];
    if (n == 0) continue;
    cudaError_t e = rows_to_device(qkv_dev + size_t(b0) * units, units,
                                   qkv_host + b0 * qkv_stride, qkv_stride, n, cs);
    if (e == cudaSuccess && rope != FA_ROPE_NONE)
      e = cudaMemcpyAsync(angles_dev + size_t(b0) * d, angles_host + int64_t(b0) * d,
                          size_t(n) * d * 4, cudaMemcpyHostToDevice, cs);
    if (e == cudaSuccess) e = cudaEventRecord(in_ready[g], cs);
    cudaStream_t gs = g % 2 == 1 ? side : s;
    if (e == cudaSuccess) e = cudaStreamWaitEvent(gs, in_ready[g], 0);
    if (e != cudaSuccess) {
      rc = cuda_fail(e, "rows to device");
      break;
    }
    rc = fa_attention_batch(caches + b0, spans + b0, n, layer, rope,
                            rope != FA_ROPE_NONE ? angles_dev + size_t(b0) * d : nullptr, norm,
                            qkv_dev + size_t(b0) * units, units, out_dev + b0 * out_dev_stride,
                            out_dev_stride, gs);
    if (rc == FA_OK) {
      e = cudaEventRecord(done[g], gs);
      if (e != cudaSuccess) rc = cuda_fail(e, "attention event");
    }
  }
  if (rc != FA_OK) {
    // earlier groups' kernels may still be storing into the caller's (mapped) output, and
    // their copies may be in flight: all of them end before the call returns its error
    cudaStreamSynchronize(s);
    cudaStreamSynchronize(side);
    cudaStreamSynchronize(cs);
    return rc;
  }
  // the caller's stream ends after the side stream's groups
  if (side != s) {
    FA_CUDA(cudaEventRecord(side_end, side), "side stream event");
    FA_CUDA(cudaStreamWaitEvent(s, side_end, 0), "stream wait");
  }
  if (out_mapped) {
    // the caller's stream ran (or waited for) every group: its end is the call's end
    FA_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    return FA_OK;
  }
  for (int g = 0; g < groups; ++g) {
    const int b0 = bounds[g], n = bounds[g + 1] - bounds[g];
    if (n == 0) continue;
    FA_CUDA(cudaStreamWaitEvent(cs, done[g], 0), "copy stream wait");
    FA_CUDA(cudaMemcpy2DAsync(out_host + b0 * out_stride, out_stride * 4,
                              out_dev + size_t(b0) * width, width * 4, width * 4, n,
                              cudaMemcpyDeviceToHost, cs),
            "out to host");
  }
  FA_CUDA(cudaStreamSynchronize(cs), "cudaStreamSynchronize");
  FA_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
  return FA_OK;
}

int fa_attend_partial(fa_kvcache* cache, int32_t layer, const float* q, int32_t key_begin,
                      int32_t key_end, float* partials, void* stream) {
  if (int rc = check_cache(cache)) return rc;
  if (int rc = check_layer(cache, layer)) return rc;
  if (q == nullptr || partials == nullptr) return fail(FA_ERR_ARG, "null q or partials");
  FA_PTR(q, cache->device);
  FA_PTR(partials, cache->device);
  if (key_begin < 0 || key_end < key_begin) return fail(FA_ERR_ARG, "key range");
  if (key_end - key_begin > cache->capacity)
    return fail(FA_ERR_CAPACITY, "%d keys in a cache of %d", key_end - key_begin, cache->capacity);
  DeviceGuard guard(cache->device);
  auto s = static_cast<cudaStream_t>(stream);
  const int64_t width = int64_t(cache->heads) * cache->head_dim;
  const int n = key_end - key_begin;
  const Plan p = plan_span(cache, 1, std::max(n, 1));
  Work w;
  if (int rc = ensure_work(cache, 0, size_t(p.chunks) * cache->heads, 0, s, &w)) return rc;
  if (int rc = ensure_counters(cache, size_t(p.kv_groups), s)) return rc;
  if (n == 0) {
    // No keys: max -inf, sum 0, o 0 for every head.
    std::vector<float> empty(size_t(cache->heads) * (cache->head_dim + 2), 0.0f);
    for (int h = 0; h < cache->heads; ++h) empty[size_t(h) * (cache->head_dim + 2)] = -INFINITY;
    FA_CUDA(cudaMemcpyAsync(partials, empty.data(), empty.size() * 4, cudaMemcpyHostToDevice, s),
            "empty partials");
    FA_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    return FA_OK;
  }
  // The range is the key run of one row at position key_end - 1 under Window(n): positions
  // key_begin .. key_end - 1, every one visible.
  fa::SpanArgs args{};
  fill_common(&args.c, cache, p);
  args.c.q = q;
  args.c.q_stride = width;
  args.c.out = nullptr;
  args.c.partial_out = partials;
  args.c.part_o = w.part_o;
  args.c.part_ml = w.part_ml;
  args.c.counters = static_cast<int*>(cache->counters.ptr);
  args.k = layer_ptr(cache, cache->keys, layer);
  args.v = layer_ptr(cache, cache->values, layer);
  args.capacity = cache->capacity;
  args.rows = 1;
  args.first = key_end - 1;
  args.end = key_end;
  args.kind = FA_MASK_WINDOW;
  args.window = n;
  args.chunks = p.chunks;
  args.c.cluster = p.cluster;
  args.rows_per_image = 1;
  args.keys_per_image = 0;
  fa::AttendLaunch l{cache->dtype == FA_F32 ? fa::kKtF32 : fa::kKtBf16, p.g, false, &args, nullptr,
                     p.kv_groups * p.chunks};
  cudaError_t e = launch_attend_d(cache->head_dim, l, s);
  if (e != cudaSuccess) return cuda_fail(e, "attend launch");
  return FA_OK;
}

int fa_merge_partials(const float* partials, int32_t shards, int32_t heads, int32_t head_dim,
                      float* out, void* stream) {
  if (partials == nullptr || out == nullptr) return fail(FA_ERR_ARG, "null argument");
  FA_PTR(partials, current_device());
  FA_PTR(out, current_device());
  if (shards < 1 || heads < 1 || head_dim < 1 || head_dim > 1024)
    return fail(FA_ERR_ARG, "shards %d heads %d head_dim %d", shards, heads, head_dim);
  cudaError_t e = fa::launch_merge_partials(partials, shards, heads, head_dim, out,
                                            static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "merge launch");
  return FA_OK;
}

int fa_peer_buffer_bytes(int32_t world, int32_t heads, int32_t head_dim, uint64_t* bytes) {
  if (bytes == nullptr) return fail(FA_ERR_ARG, "null bytes");
  if (world < 1 || world > fa::kMaxPeers || heads < 1 || heads > fa::kMaxPeerHeads ||
      head_dim < 1 || head_dim > 1024)
    return fail(FA_ERR_ARG, "world %d (1..%d), heads %d (1..%d), head_dim %d", world,
                fa::kMaxPeers, heads, fa::kMaxPeerHeads, head_dim);
  *bytes = fa::peer_buffer_bytes(world, heads, head_dim);
  return FA_OK;
}

int fa_peer_alloc(uint64_t bytes, void** ptr, fa_ipc_handle* handle) {
  if (ptr == nullptr || handle == nullptr || bytes < uint64_t(fa::kPeerHeaderBytes))
    return fail(FA_ERR_ARG, "null argument or a buffer below its header");
  void* p = nullptr;
  FA_CUDA(cudaMalloc(&p, bytes), "cudaMalloc(peer buffer)");
  cudaError_t e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "peer buffer");
  }
  static_assert(sizeof(h) == sizeof(handle->bytes), "a CUDA IPC handle is 64 bytes");
  std::memcpy(handle->bytes, &h, sizeof(h));
  *ptr = p;
  return FA_OK;
}

int fa_peer_open(const fa_ipc_handle* handle, void** ptr) {
  if (handle == nullptr || ptr == nullptr) return fail(FA_ERR_ARG, "null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof(h));
  FA_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return FA_OK;
}

int fa_peer_close(void* ptr) {
  if (ptr == nullptr) return FA_OK;
  FA_CUDA(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
  return FA_OK;
}

int fa_peer_free(void* ptr) {
  if (ptr == nullptr) return FA_OK;
  FA_CUDA(cudaFree(ptr), "cudaFree(peer buffer)");
  return FA_OK;
}

int fa_peer_reset(void* own_buffer, uint64_t buffer_bytes, void* stream) {
  if (own_buffer == nullptr) return fail(FA_ERR_ARG, "null buffer");
  if (buffer_bytes < uint64_t(fa::kPeerHeaderBytes)) return fail(FA_ERR_ARG, "a buffer below its header");
  FA_PTR(own_buffer, current_device());
  auto s = static_cast<cudaStream_t>(stream);
  // the step counter and every stamped word: no word of an earlier step can match a new one
  FA_CUDA(cudaMemsetAsync(own_buffer, 0, buffer_bytes, s), "clear exchange buffer");
  FA_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
  return FA_OK;
}

int fa_exchange_merge(void* const* buffers, uint64_t buffer_bytes, int32_t rank, int32_t world,
                      int32_t heads, int32_t head_dim, const float* partials, float* out,
                      void* stream) {
  uint64_t need = 0;
  if (int rc = fa_peer_buffer_bytes(world, heads, head_dim, &need)) return rc;
  if (buffers == nullptr || partials == nullptr || out == nullptr)
    return fail(FA_ERR_ARG, "null argument");
  if (rank < 0 || rank >= world) return fail(FA_ERR_ARG, "rank %d of %d", rank, world);
  if (buffer_bytes < need)
    return fail(FA_ERR_SHAPE, "exchange buffers of %llu bytes, %llu needed",
                (unsigned long long)buffer_bytes, (unsigned long long)need);
  const int device = current_device();
  FA_PTR(partials, device);
  FA_PTR(out, device);
  fa::PeerMergeArgs a{};
  for (int r = 0; r < world; ++r) {
    if (buffers[r] == nullptr) return fail(FA_ERR_ARG, "no buffer for rank %d", r);
    a.bufs[r] = static_cast<unsigned char*>(buffers[r]);
  }
  Device* dev = nullptr;
  if (int rc = device_state(device, &dev)) return rc;
  a.rank = rank;
  a.world = world;
  a.heads = heads;
  a.head_dim = head_dim;
  a.partials = partials;
  a.out = out;
  a.err = dev->err;
  cudaError_t e = fa::launch_peer_merge(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "exchange launch");
  return FA_OK;
}

int fa_attend_full(const fa_call* call, void* out, int64_t out_stride, void* stream) {
  if (call == nullptr || out == nullptr) return fail(FA_ERR_ARG, "null argument");
  const fa_call& k = *call;
  if (k.heads < 1 || k.kv_heads < 1 || k.images < 0 || k.queries < 0 || k.keys < 0)
    return fail(FA_ERR_ARG, "call sizes");
  if (k.heads % k.kv_heads != 0) return fail(FA_ERR_SHAPE, "%d heads over %d KV heads", k.heads, k.kv_heads);
  if (!supported_head_dim(k.head_dim, k.dtype)) return fail(FA_ERR_UNSUPPORTED, "head_dim %d", k.head_dim);
  if (k.dtype != FA_F32 && k.dtype != FA_BF16) return fail(FA_ERR_ARG, "dtype %d", k.dtype);
  if (k.out_dtype != FA_F32 && k.out_dtype != FA_BF16)
    return fail(FA_ERR_ARG, "output dtype %d", k.out_dtype);
  if (k.images == 0 || k.queries == 0) return FA_OK;
  if (k.keys == 0) return fail(FA_ERR_ARG, "a full-mask call without keys");
  if (k.query.values == nullptr || k.key.values == nullptr || k.value.values == nullptr)
    return fail(FA_ERR_ARG, "null operand");
  FA_PTR(k.query.values, current_device());
  FA_PTR(k.key.values, current_device());
  FA_PTR(k.value.values, current_device());
  FA_PTR(out, current_device());
  const int64_t width = int64_t(k.heads) * k.head_dim;
  if (out_stride < width) return fail(FA_ERR_SHAPE, "output rows narrower than heads x head_dim");
  const size_t esize = k.dtype == FA_F32 ? 4 : 2;
  const int64_t align = 16 / int64_t(esize);
  if (k.key.stride % align || k.key.offset % align || k.value.stride % align ||
      k.value.offset % align || k.key.stride != k.value.stride ||
      reinterpret_cast<uintptr_t>(k.key.values) % 16 || reinterpret_cast<uintptr_t>(k.value.values) % 16)
    return fail(FA_ERR_UNSUPPORTED, "key/value rows must start on 16-byte boundaries with one stride");
  int device = 0;
  FA_CUDA(cudaGetDevice(&device), "cudaGetDevice");
  Device* dev = nullptr;
  if (int rc = device_state(device, &dev)) return rc;
  auto s = static_cast<cudaStream_t>(stream);
  const size_t oesize = k.out_dtype == FA_F32 ? 4 : 2;
  const bool tma_ok = k.query.stride % align == 0 && k.query.offset % align == 0 &&
                      reinterpret_cast<uintptr_t>(k.query.values) % 16 == 0 &&
                      (out_stride * int64_t(oesize)) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(out) % 16 == 0;
  if (tma_ok && fa::fmha_supported(k.dtype == FA_BF16, k.head_dim)) {
    fa::FmhaArgs a{};
    a.heads = k.heads;
    a.kv_heads = k.kv_heads;
    a.group = k.heads / k.kv_heads;
    a.rows = k.queries;
    a.images = k.images;
    a.q_tiles = (k.queries + 127) / 128;
    a.first = 0;
    a.end = k.keys;
    a.kind = FA_MASK_FULL;
    a.q_row_base_per_image = k.queries;
    a.kv_row_base_per_image = k.keys;
    a.kv_layer_base = 0;
    a.scale_log2 = query_scale(k.head_dim);
    a.out = out;
    a.out_stride = out_stride;
    a.out_bf16 = k.out_dtype == FA_BF16 ? 1 : 0;
    a.err = dev->err;
    a.band_heads = band_heads(k.heads, k.kv_heads,
                              2.0 * k.images * double(k.keys) * k.head_dim * (k.dtype == FA_BF16 ? 2 : 4));
    if (fa::fmha_splits_supported(k.dtype == FA_BF16, k.head_dim)) {
      const int64_t units = int64_t(k.images) * ((a.q_tiles + 1) / 2) * k.heads;
      int64_t whole = units;
      int splits = 1;
      plan_full_split(units, dev->sms, (k.keys + 127) / 128, &whole, &splits);
      const size_t tail = size_t(units - whole);
      const size_t o_bytes = align_up(tail * splits * 256 * k.head_dim * 4, 256);
      const size_t ml_bytes = align_up(tail * splits * 256 * 2 * 4, 256);
      if (splits > 1 && o_bytes + ml_bytes <= kMaxSplitBytes) {
        std::lock_guard<std::mutex> lock(g_split_mutex);
        SplitWork& w = g_split_work[{device, s}];
        if (int rc = w.partials.ensure(o_bytes + ml_bytes, s)) return rc;
        const int epoch = dev->epoch.load();
        if (tail * 8 * sizeof(int) > w.counters.bytes || w.counters_epoch != epoch) {
          if (int rc = w.counters.ensure(tail * 8 * sizeof(int), s)) return rc;
          FA_CUDA(cudaMemsetAsync(w.counters.ptr, 0, w.counters.bytes, s), "clear split counters");
          w.counters_epoch = epoch;
        }
        a.whole_units = int(whole);
        a.splits = splits;
        a.part_o = static_cast<float*>(w.partials.ptr);
        a.part_ml = reinterpret_cast<float*>(static_cast<unsigned char*>(w.partials.ptr) + o_bytes);
        a.counters = static_cast<int*>(w.counters.ptr);
      }
    }
    fa::FmhaLaunch l{k.dtype == FA_BF16 ? 1 : 0, k.head_dim,
                     static_cast<const unsigned char*>(k.query.values) + k.query.offset * esize,
                     uint64_t(k.images) * k.queries, uint64_t(k.heads), uint64_t(k.query.stride),
                     uint64_t(k.head_dim),
                     static_cast<const unsigned char*>(k.key.values) + k.key.offset * esize,
                     static_cast<const unsigned char*>(k.value.values) + k.value.offset * esize,
                     uint64_t(k.images) * k.keys, uint64_t(k.kv_heads), uint64_t(k.key.stride),
                     uint64_t(k.head_dim), a};
    cudaError_t e = fa::launch_fmha(l, s);
    if (e != cudaSuccess) return cuda_fail(e, "tensor-core attention launch");
    return FA_OK;
  }
  if (k.out_dtype != FA_F32)
    return fail(FA_ERR_UNSUPPORTED, "bf16 output needs the tensor-core path (head_dim 64/128, "
                                    "16-byte aligned rows)");
  // A call-local workspace, kept per (device, stream) and grown on demand: calls on one stream
  // run in order and share it, calls on different streams do not.
  const int rows = k.images * k.queries;
  fa_kvcache view;  // the call viewed as a cache for the planner
  view.layers = 1;
  view.heads = k.heads;
  view.kv_heads = k.kv_heads;
  view.head_dim = k.head_dim;
  view.capacity = k.images * k.keys;
  view.dtype = k.dtype;
  view.device = device;
  view.dev = dev;
  const Plan p = plan_span(&view, rows, k.keys);
  const size_t q_bytes = align_up(size_t(rows) * width * 4, 256);
  const size_t o_bytes = align_up(size_t(rows) * p.chunks * k.heads * kernel_dim(k.head_dim) * 4, 256);
  const size_t ml_bytes = align_up(size_t(rows) * p.chunks * k.heads * 2 * 4, 256);
  std::unique_lock<std::mutex> lock(g_split_mutex);
  SplitWork& fw = g_full_work[{device, s}];
  if (int rc = fw.partials.ensure(q_bytes + o_bytes + ml_bytes, s)) return rc;
  const size_t counter_bytes = size_t(rows) * p.kv_groups * sizeof(int);
  if (counter_bytes > fw.counters.bytes || fw.counters_epoch != dev->epoch.load()) {
    if (int rc = fw.counters.ensure(counter_bytes, s)) return rc;
    FA_CUDA(cudaMemsetAsync(fw.counters.ptr, 0, fw.counters.bytes, s), "counters");
    fw.counters_epoch = dev->epoch.load();
  }
  unsigned char* base = static_cast<unsigned char*>(fw.partials.ptr);
  int* counter_base = static_cast<int*>(fw.counters.ptr);
  lock.unlock();
  float* q = reinterpret_cast<float*>(base);
  cudaError_t e = fa::launch_prepare_queries(k.dtype, k.query.values, k.query.stride, k.query.offset,
                                             rows, k.heads, k.head_dim, query_scale(k.head_dim), q, s);
  if (e != cudaSuccess) return cuda_fail(e, "query scaling");
  fa::SpanArgs args{};
  args.c.heads = k.heads;
  args.c.kv_heads = k.kv_heads;
  args.c.group = k.heads / k.kv_heads;
  args.c.hgroups = p.hgroups;
  args.c.kv_stride = k.head_dim;  // KV head h at h * head_dim within a row
  args.c.key_stride = k.key.stride;
  args.c.q_scale = 1.0f;  // prepare_queries scaled them
  args.c.err = dev->err;
  args.c.dh = k.head_dim;
  args.c.q = q;
  args.c.q_stride = width;
  args.c.out = static_cast<float*>(out);
  args.c.out_stride = out_stride;
  args.c.part_o = reinterpret_cast<float*>(base + q_bytes);
  args.c.part_ml = reinterpret_cast<float*>(base + q_bytes + o_bytes);
  args.c.counters = counter_base;
  args.k = static_cast<const unsigned char*>(k.key.values) + k.key.offset * esize;
  args.v = static_cast<const unsigned char*>(k.value.values) + k.value.offset * esize;
  args.capacity = INT_MAX;
  args.rows = rows;
  args.first = 0;
  args.end = k.keys;
  args.kind = FA_MASK_FULL;
  args.chunks = p.chunks;
  args.c.cluster = p.cluster;
  args.rows_per_image = k.queries;
  args.keys_per_image = k.keys;
  fa::AttendLaunch l{k.dtype == FA_F32 ? fa::kKtF32 : fa::kKtBf16, p.g, false, &args, nullptr,
                     rows * p.kv_groups * p.chunks};
  e = launch_attend_d(k.head_dim, l, s);
  if (e != cudaSuccess) return cuda_fail(e, "attend launch");
  return FA_OK;
}

int fa_attend_relpos(const fa_relpos_call* call, float* out, int64_t out_stride, void* stream) {
  if (call == nullptr || out == nullptr) return fail(FA_ERR_ARG, "null argument");
  const fa_relpos_call& c = *call;
  if (c.heads < 1 || c.frames < 0) return fail(FA_ERR_ARG, "heads %d frames %d", c.heads, c.frames);
  if (c.head_dim != 32 && c.head_dim != 64 && c.head_dim != 128 && c.head_dim != 256)
    return fail(FA_ERR_UNSUPPORTED, "relative-position attention with head_dim %d", c.head_dim);
  if (c.frames == 0) return FA_OK;
  if (c.query.values == nullptr || c.key.values == nullptr || c.value.values == nullptr ||
      c.positions == nullptr || c.bias_u == nullptr || c.bias_v == nullptr)
    return fail(FA_ERR_ARG, "null operand");
  const int64_t width = int64_t(c.heads) * c.head_dim;
  if (c.key.stride != c.value.stride) return fail(FA_ERR_ARG, "keys and values need one stride");
  if (c.query.stride < width || c.key.stride < width || c.positions_stride < width ||
      out_stride < width)
    return fail(FA_ERR_SHAPE, "rows narrower than heads x head_dim");
  const int device = current_device();
  FA_PTR(c.query.values, device);
  FA_PTR(c.key.values, device);
  FA_PTR(c.value.values, device);
  FA_PTR(c.positions, device);
  FA_PTR(c.bias_u, device);
  FA_PTR(c.bias_v, device);
  FA_PTR(out, device);
  fa::RelposArgs a{};
  a.heads = c.heads;
  a.frames = c.frames;
  a.q = static_cast<const float*>(c.query.values) + c.query.offset;
  a.q_stride = c.query.stride;
  a.k = static_cast<const float*>(c.key.values) + c.key.offset;
  a.v = static_cast<const float*>(c.value.values) + c.value.offset;
  a.kv_stride = c.key.stride;
  a.positions = c.positions;
  a.positions_stride = c.positions_stride;
  a.bias_u = c.bias_u;
  a.bias_v = c.bias_v;
  a.scale_log2 = query_scale(c.head_dim);
  a.out = out;
  a.out_stride = out_stride;
  const cudaError_t e = fa::launch_relpos(a, c.head_dim, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "relative-position attention launch");
  return FA_OK;
}

int fa_normalize_and_rotate(const fa_prologue* prologue, const float* qkv, int64_t qkv_stride,
                            void* out, int64_t out_stride, int32_t out_dtype, void* stream) {
  if (prologue == nullptr) return fail(FA_ERR_ARG, "null prologue");
  const fa_prologue& p = *prologue;
  if (p.tokens < 0 || p.heads < 1 || p.head_dim < 2 || p.head_dim > 256 || p.head_dim % 2 != 0)
    return fail(FA_ERR_ARG, "tokens %d heads %d head_dim %d", p.tokens, p.heads, p.head_dim);
  if (p.norm < FA_NORM_NONE || p.norm > FA_NORM_HEAD) return fail(FA_ERR_ARG, "norm %d", p.norm);
  if (int rc = check_rope(p.rope, p.angles)) return rc;
  if (out_dtype != FA_F32 && out_dtype != FA_BF16) return fail(FA_ERR_ARG, "out dtype %d", out_dtype);
  if (p.tokens == 0) return FA_OK;
  if (qkv == nullptr || out == nullptr) return fail(FA_ERR_ARG, "null qkv or out");
  if (p.norm != FA_NORM_NONE && (p.q_norm == nullptr || p.k_norm == nullptr))
    return fail(FA_ERR_ARG, "norm without weights");
  const int64_t width = int64_t(p.heads) * p.head_dim;
  if (qkv_stride < 3 * width || out_stride < 3 * width)
    return fail(FA_ERR_SHAPE, "rows narrower than queries, keys and values");
  const bool in_place = out == static_cast<const void*>(qkv);
  if (in_place && (out_dtype != FA_F32 || out_stride != qkv_stride))
    return fail(FA_ERR_ARG, "in place needs FA_F32 and one stride");
  const int device = current_device();
  FA_PTR(qkv, device);
  FA_PTR(out, device);
  FA_PTR(p.q_norm, device);
  FA_PTR(p.k_norm, device);
  FA_PTR(p.angles, device);
  fa::PrologueArgs a{};
  a.tokens = p.tokens;
  a.heads = p.heads;
  a.head_dim = p.head_dim;
  a.norm = p.norm;
  a.rope = p.rope;
  a.rotated_rows = p.rope == FA_ROPE_NONE ? 0 : std::max(0, std::min(p.rotated_rows, p.tokens));
  a.parts = in_place ? 2 : 3;
  a.vec_in = reinterpret_cast<uintptr_t>(qkv) % 16 == 0 && qkv_stride % 4 == 0 && width % 4 == 0;
  const int out_elem = out_dtype == FA_F32 ? 4 : 2;
  a.vec_out = reinterpret_cast<uintptr_t>(out) % 16 == 0 && (out_stride * out_elem) % 16 == 0 &&
              width % 4 == 0;
  a.out_bf16 = out_dtype == FA_BF16 ? 1 : 0;
  a.qkv = qkv;
  a.qkv_stride = qkv_stride;
  a.q_norm = p.q_norm;
  a.k_norm = p.k_norm;
  a.eps = p.eps;
  a.angles = p.angles;
  a.out = out;
  a.out_stride = out_stride;
  Device* dev = nullptr;
  if (int rc = device_state(device, &dev)) return rc;
  a.err = dev->err;
  const cudaError_t e = fa::launch_prologue(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "prologue launch");
  return FA_OK;
}

int fa_gated_attention(fa_kvcache* cache, int32_t layer, const fa_span* span, int32_t gate,
                       int32_t rotary_dim, const float* angles, const fa_head_norm* norm,
                       const float* qkv, int64_t qkv_stride, float* out, int64_t out_stride,
                       void* stream) {
  if (int rc = check_cache(cache)) return rc;
  if (int rc = check_layer(cache, layer)) return rc;
  std::vector<int> ends;
  if (int rc = check_span(cache, span, &ends)) return rc;
  if (gate < FA_GATE_NONE || gate > FA_GATE_HEADWISE) return fail(FA_ERR_ARG, "gate %d", gate);
  const int d = cache->head_dim;
  if (rotary_dim < 2 || rotary_dim > d || rotary_dim % 2 != 0)
    return fail(FA_ERR_ARG, "rotary_dim %d of head_dim %d", rotary_dim, d);
  if (int rc = check_rope(FA_ROPE_HALF, angles)) return rc;
  const int gate_heads = gate == FA_GATE_ELEMENTWISE ? cache->heads : 0;
  const int64_t head_columns = int64_t(cache->heads + gate_heads + 2 * cache->kv_heads) * d;
  const int64_t columns = head_columns + (gate == FA_GATE_HEADWISE ? cache->heads : 0);
  const int64_t width = int64_t(cache->heads) * d;
  if (span->rows > 0 && (qkv == nullptr || out == nullptr)) return fail(FA_ERR_ARG, "null qkv or out");
  FA_PTR(qkv, cache->device);
  FA_PTR(angles, cache->device);
  FA_PTR(out, cache->device);
  if (qkv_stride < columns || out_stride < width)
    return fail(FA_ERR_SHAPE, "row strides below the heads' widths");
  if (span->rows == 0) return FA_OK;
  DeviceGuard guard(cache->device);
  auto s = static_cast<cudaStream_t>(stream);
  Work w;
  int rc = FA_OK;
  if (span_on_tensor_cores(cache, span)) {
    if ((rc = ensure_work(cache, size_t(span->rows) * width, 0, 0, s, &w))) return rc;
    if ((rc = rope_rows(cache, layer, span, FA_ROPE_HALF, angles, norm, qkv, qkv_stride, w.q,
                        width, 1.0f, true, s, cache->dtype == FA_BF16, gate_heads, rotary_dim)))
      return rc;
    rc = attend_rows_tc(cache, layer, span, ends, w.q, width, out, out_stride, s);
  } else if (std::vector<fa::Runs> truns; span_decode_tc(cache, span, ends, &truns)) {
    const DtcPlan plan = plan_decode_tc(cache, truns, span->rows);
    if ((rc = ensure_work(cache, size_t(span->rows) * width, size_t(plan.slots) * cache->heads, 0,
                          s, &w)))
      return rc;
    if ((rc = rope_rows(cache, layer, span, FA_ROPE_HALF, angles, norm, qkv, qkv_stride, w.q,
                        width, 1.0f, true, s, false, gate_heads, rotary_dim)))
      return rc;
    std::vector<fa_kvcache*> same(span->rows, cache);
    rc = attend_batch_tc(same.data(), truns, span->rows, layer, w.q, width, out, out_stride, s, &w);
  } else {
    const Plan pl = plan_for_span(cache, span, ends);
    if ((rc = ensure_work(cache, size_t(span->rows) * width,
                          size_t(span->rows) * pl.chunks * cache->heads, 0, s, &w)))
      return rc;
    if ((rc = rope_rows(cache, layer, span, FA_ROPE_HALF, angles, norm, qkv, qkv_stride, w.q,
                        width, 1.0f, true, s, false, gate_heads, rotary_dim)))
      return rc;
    rc = attend_rows(cache, layer, span, ends, pl, w, w.q, width, out, out_stride, nullptr, s);
  }
  if (rc != FA_OK || gate == FA_GATE_NONE) return rc;
  fa::GateArgs g{};
  g.rows = span->rows;
  g.heads = cache->heads;
  g.head_dim = d;
  g.per_head = gate == FA_GATE_HEADWISE ? 1 : 0;
  g.qkv = qkv;
  g.qkv_stride = qkv_stride;
  g.gate_offset = gate == FA_GATE_HEADWISE ? head_columns : width;
  g.out = out;
  g.out_stride = out_stride;
  const cudaError_t e = fa::launch_gate(g, s);
  if (e != cudaSuccess) return cuda_fail(e, "gate launch");
  return FA_OK;
}

int fa_device_status(void* stream) {
  int device = 0;
  FA_CUDA(cudaGetDevice(&device), "cudaGetDevice");
  Device* dev = nullptr;
  if (int rc = device_state(device, &dev)) return rc;
  FA_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "cudaStreamSynchronize");
  unsigned word = 0;
  FA_CUDA(cudaMemcpy(&word, dev->err, sizeof word, cudaMemcpyDeviceToHost), "read error word");
  if (word != 0) {
    FA_CUDA(cudaMemset(dev->err, 0, sizeof word), "clear error word");
    dev->epoch.fetch_add(1);
    return fail(FA_ERR_TIMEOUT, "a device-side wait gave up (error word 0x%x)", word);
  }
  return FA_OK;
}

int fa_rng_fill_normal(uint64_t seed, float* out, int64_t n) {
  if (n < 0 || (n > 0 && out == nullptr)) return fail(FA_ERR_ARG, "bad output");
  // SplitMix64 seeding of xoshiro256** (rng.rs:10-35).
  uint64_t mixed = seed;
  auto next_seed = [&]() {
    mixed += 0x9E3779B97F4A7C15ull;
    uint64_t z = mixed;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  };
  uint64_t st[4] = {next_seed(), next_seed(), next_seed(), next_seed()};
  auto rotl = [](uint64_t x, int k) { return (x << k) | (x >> (64 - k)); };
  auto next = [&]() {
    const uint64_t result = rotl(st[1] * 5, 7) * 9;
    const uint64_t t = st[1] << 17;
    st[2] ^= st[0];
    st[3] ^= st[1];
    st[1] ^= st[2];
    st[0] ^= st[3];
    st[2] ^= t;
    st[3] = rotl(st[3], 45);
    return result;
  };
  // Uniform in (0, 1] (rng.rs:37-40); Box-Muller pairs (rng.rs:42-52).
  auto uniform = [&]() { return double((next() >> 11) + 1) / double(1ull << 53); };
  const double tau = 6.283185307179586476925286766559;
  for (int64_t i = 0; i < n; i += 2) {
    const double radius = std::sqrt(-2.0 * std::log(uniform()));
    const double angle = tau * uniform();
    out[i] = float(radius * std::cos(angle));
    if (i + 1 < n) out[i + 1] = float(radius * std::sin(angle));
  }
  return FA_OK;
}

}  // extern "C"

// ---- fa_attend_static: KvCache::attend without allocating ----------------------------------
//
// Some callers cannot allocate device memory at call time: a host that pre-reserves all of the
// GPU's memory for its own pool (another framework's caching allocator, or an embedding runtime
// with a fixed memory budget) has none left for cudaMalloc, and a latency-bound decode loop
// cannot afford cudaMalloc's implicit device synchronisation when a span first outgrows the
// cache's workspace. fa_attend_static serves them: the split-KV partials and arrival counters
// of the attention live in one file-scope device array, the caller passes only its queries and
// output. That array is kStaticScratchBytes on every GPU that loads the library, held until the
// process exits.
namespace {

constexpr size_t kStaticScratchBytes = size_t(4) << 20;   // 4 MiB per device
constexpr size_t kStaticCounterBytes = size_t(64) << 10;  // its first 64 KiB: arrival counters

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// The array's device address, per device; in host code g_static_scratch names a host-side
// stand-in, not device memory, so it is looked up once per device with that device current.
constexpr int kStaticScratchDevices = 64;
unsigned char* g_static_scratch_addr[kStaticScratchDevices];
std::mutex g_static_scratch_mutex;

// Called with `device` current (the caller's DeviceGuard).
int static_scratch_address(int device, unsigned char** out) {
  if (device < 0 || device >= kStaticScratchDevices)
    return fail(FA_ERR_ARG, "device %d: fa_attend_static serves devices 0..%d", device,
                kStaticScratchDevices - 1);
  std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
  if (g_static_scratch_addr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
    g_static_scratch_addr[device] = static_cast<unsigned char*>(p);
  }
  *out = g_static_scratch_addr[device];
  return FA_OK;
}

}  // namespace

extern "C" int fa_attend_static(fa_kvcache* cache, int32_t layer, const fa_span* span,
                                const float* q, int64_t q_stride, float* out, int64_t out_stride,
                                void* stream) {
  if (int rc = check_cache(cache)) return rc;
  if (int rc = check_layer(cache, layer)) return rc;
  if (span == nullptr) return fail(FA_ERR_ARG, "null span");
  if (span->rows < 0 || span->first < 0) return fail(FA_ERR_ARG, "negative span");
  const fa_mask& m = span->mask;
  if (m.kind < FA_MASK_CAUSAL || m.kind > FA_MASK_GROUPS) return fail(FA_ERR_ARG, "mask kind %d", m.kind);
  if (m.kind == FA_MASK_WINDOW && m.window < 1) return fail(FA_ERR_ARG, "window %d", m.window);
  const int64_t end = int64_t(span->first) + span->rows;
  const int64_t reach = m.kind == FA_MASK_WINDOW ? int64_t(m.window) + span->rows : end;
  if (reach > cache->capacity)
    return fail(FA_ERR_CAPACITY, "the cache holds every key the span sees: %lld > capacity %d",
                (long long)reach, cache->capacity);
  // Groups ends into a fixed array: nothing on this path allocates, on the host either.
  int ends[fa::kMaxEnds];
  int n_ends = 0;
  if (m.kind == FA_MASK_GROUPS) {
    if (m.n_ends < 1 || m.ends == nullptr || m.n_ends > fa::kMaxEnds)
      return fail(FA_ERR_ARG, "Groups needs 1..%d ends", fa::kMaxEnds);
    if (m.state < 0 || m.state > end) return fail(FA_ERR_ARG, "Groups state %d", m.state);
    for (int i = 0; i < m.n_ends; ++i) {
      if (m.ends[i] <= (i == 0 ? m.state - 1 : m.ends[i - 1]) || m.ends[i] > end)
        return fail(FA_ERR_ARG, "Groups ends must rise after the state and end by the call's end");
      ends[n_ends++] = m.ends[i];
    }
    if (ends[n_ends - 1] != end) return fail(FA_ERR_ARG, "the last group ends with the call");
  }
  const int64_t width = int64_t(cache->heads) * cache->head_dim;
  if (span->rows == 0) return FA_OK;
  if (q == nullptr || out == nullptr) return fail(FA_ERR_ARG, "null q or out");
  FA_PTR(q, cache->device);
  FA_PTR(out, cache->device);
  if (q_stride < width || out_stride < width)
    return fail(FA_ERR_SHAPE, "row strides below heads x head_dim");
  // The split of fa_attend's split-KV kernel, and the scratch it needs.
  int max_keys = 0;
  for (int r = 0; r < span->rows; ++r) {
    const fa::Runs runs = fa::mask_runs(m.kind, m.window, m.state, n_ends, ends,
                                        span->first + r, int(end));
    max_keys = std::max(max_keys, runs.n0 + runs.n1);
  }
  const Plan p = plan_span(cache, span->rows, max_keys);
  const size_t counter_bytes = size_t(span->rows) * p.kv_groups * sizeof(int);
  const size_t slots = size_t(span->rows) * p.chunks * cache->heads;
  const size_t o_bytes = align_up(slots * kernel_dim(cache->head_dim) * 4, 256);
  const size_t ml_bytes = align_up(slots * 2 * 4, 256);
  if (counter_bytes > kStaticCounterBytes ||
      o_bytes + ml_bytes > kStaticScratchBytes - kStaticCounterBytes)
    return fail(FA_ERR_ARG,
                "this span needs %zu bytes of split-KV scratch (%d rows x %d chunks x %d heads); "
                "fa_attend_static holds %zu: use fa_attend",
                counter_bytes + o_bytes + ml_bytes, span->rows, p.chunks, cache->heads,
                kStaticScratchBytes);
  DeviceGuard guard(cache->device);
  auto s = static_cast<cudaStream_t>(stream);
  unsigned char* scratch = nullptr;
  if (int rc = static_scratch_address(cache->device, &scratch)) return rc;
  // The counters must start at zero; the array keeps whatever the last call left there.
  FA_CUDA(cudaMemsetAsync(scratch, 0, counter_bytes, s), "clear static counters");
  fa::SpanArgs args{};
  fill_common(&args.c, cache, p);
  args.c.q = q;
  args.c.q_stride = q_stride;
  args.c.out = out;
  args.c.out_stride = out_stride;
  args.c.partial_out = nullptr;
  args.c.counters = reinterpret_cast<int*>(scratch);
  args.c.part_o = reinterpret_cast<float*>(scratch + kStaticCounterBytes);
  args.c.part_ml = reinterpret_cast<float*>(scratch + kStaticCounterBytes + o_bytes);
  args.k = layer_ptr(cache, cache->keys, layer);
  args.v = layer_ptr(cache, cache->values, layer);
  args.capacity = cache->capacity;
  args.rows = span->rows;
  args.first = span->first;
  args.end = int(end);
  args.kind = m.kind;
  args.window = m.window;
  args.state = m.state;
  args.n_ends = n_ends;
  args.chunks = p.chunks;
  args.c.cluster = p.cluster;
  args.rows_per_image = span->rows;
  args.keys_per_image = 0;
  for (int i = 0; i < n_ends; ++i) args.ends[i] = ends[i];
  fa::AttendLaunch l{cache->dtype == FA_F32 ? fa::kKtF32 : fa::kKtBf16, p.g, false, &args, nullptr,
                     span->rows * p.kv_groups * p.chunks};
  const cudaError_t e = launch_attend_d(cache->head_dim, l, s);
  if (e != cudaSuccess) return cuda_fail(e, "attend launch");
  return FA_OK;
}
