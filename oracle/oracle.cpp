// CPU oracle for the attention hot path -- TEST INFRASTRUCTURE ONLY (see oracle.h).
//
// Build with -ffp-contract=off: the reference never fuses a multiply and an add on this path
// (Rust does not contract), and the Scalar backend's sums run in index order.
#include "oracle.h"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstring>
#include <functional>
#include <thread>
#include <vector>

namespace {

// std::f32::consts::LOG2_E and LN_2 rounded to f32.
constexpr float kLog2E = 1.44269504088896340736f;
constexpr float kLn2 = 0.693147180559945309417f;
// crates/kernels/src/ops.rs:98-114: the clamp range, ln 2 in two parts, the Cephes expf
// polynomial (highest degree first) and f32's exponent bias.
constexpr float kExpMin = -87.0f;
constexpr float kExpMax = 88.0f;
constexpr float kLn2High = 0.6933594f;
constexpr float kLn2Low = -2.1219444e-4f;
constexpr float kExpPoly[6] = {1.9875691e-4f, 1.3981999e-3f, 8.333452e-3f,
                               4.1665796e-2f, 0.16666666f,   0.5f};
constexpr int kExpBias = 127;
// ops.rs:135: exp_fast's degree-4 Taylor polynomial.
constexpr float kExpTaylor[5] = {1.0f / 24.0f, 1.0f / 6.0f, 0.5f, 1.0f, 1.0f};
// arch/mod.rs:46: values per run of exp_sweep.
constexpr int kExpRun = 8;

float from_bits(uint32_t bits) {
  float value;
  std::memcpy(&value, &bits, sizeof value);
  return value;
}

uint32_t to_bits(float value) {
  uint32_t bits;
  std::memcpy(&bits, &value, sizeof bits);
  return bits;
}

// Rust's f32::clamp (NaN passes through).
float clampf(float x, float lo, float hi) {
  if (x < lo) return lo;
  if (x > hi) return hi;
  return x;
}

// Rust's f32::max: a NaN operand yields the other.
float maxf(float a, float b) { return std::fmax(a, b); }

// round_ties_even under the default rounding mode.
float round_even(float x) { return std::nearbyint(x); }

// A minimal persistent thread team with one broadcast per run and static shares, as
// crates/team/src/team.rs:46-129 (rayon broadcast, Ctx::split, spin-then-yield barrier).
class Team {
 public:
  explicit Team(int threads) : threads_(std::max(threads, 1)) {
    for (int i = 1; i < threads_; ++i) workers_.emplace_back([this, i] { loop(i); });
  }
  ~Team() {
    stop_.store(true, std::memory_order_release);
    generation_.fetch_add(1, std::memory_order_acq_rel);
    for (auto& worker : workers_) worker.join();
  }
  int threads() const { return threads_; }

  // Runs task(index, count) on every thread and returns when all are done.
  void run(const std::function<void(int, int)>& task) {
    task_ = &task;
    done_.store(0, std::memory_order_release);
    generation_.fetch_add(1, std::memory_order_acq_rel);
    task(0, threads_);
    wait_done();
  }

  // Ctx::split (team.rs:88-93): this thread's share of 0..total in whole units of align.
  static std::pair<int64_t, int64_t> split(int64_t total, int64_t align, int index, int count) {
    int64_t units = total / align;
    int64_t start = units * index / count;
    int64_t end = units * (index + 1) / count;
    return {start * align, end * align};
  }

 private:
  void loop(int index) {
    uint64_t seen = 0;
    for (;;) {
      uint32_t spins = 0;
      uint64_t now;
      while ((now = generation_.load(std::memory_order_acquire)) == seen) {
        // Spin, then yield (team.rs:104-129); an idle team sleeps so that it does not hold the
        // host cores while a GPU benchmark runs beside it.
        if (++spins > 4096) {
          if (spins > (1u << 20)) std::this_thread::sleep_for(std::chrono::microseconds(200));
          else std::this_thread::yield();
        }
      }
      seen = now;
      if (stop_.load(std::memory_order_acquire)) return;
      (*task_)(index, threads_);
      done_.fetch_add(1, std::memory_order_acq_rel);
    }
  }
  void wait_done() {
    uint32_t spins = 0;
    while (done_.load(std::memory_order_acquire) != threads_ - 1) {
      if (++spins > 4096) std::this_thread::yield();
    }
  }

  int threads_;
  std::vector<std::thread> workers_;
  std::atomic<uint64_t> generation_{0};
  std::atomic<int> done_{0};
  std::atomic<bool> stop_{false};
  const std::function<void(int, int)>* task_ = nullptr;
};

Team* current_team = nullptr;

Team& team(int threads) {
  if (current_team == nullptr || current_team->threads() != threads) {
    delete current_team;
    current_team = new Team(threads);
  }
  return *current_team;
}

// KvCache::attend's body for one head (transformer.rs:196-218).
void attend_head(const oracle_cache* cache, int64_t layer, int64_t rows, int64_t first,
                 const oracle_mask* mask, const float* qkv, int64_t stride, float* out,
                 int64_t head, std::vector<float>& scores, std::vector<const float*>& key_rows,
                 std::vector<const float*>& value_rows) {
  const int64_t d = cache->head_dim;
  const int64_t kv_head = head / (cache->heads / cache->kv_heads);
  const int64_t width = cache->heads * d;
  for (int64_t row = 0; row < rows; ++row) {
    const int64_t position = first + row;
    int64_t runs[4];
    oracle_mask_keys(mask, position, first + rows, runs);
    const int64_t run_len = runs[1] - runs[0];
    const int64_t keys = run_len + (runs[3] - runs[2]);
    key_rows.resize(keys);
    value_rows.resize(keys);
    for (int64_t j = 0; j < keys; ++j) {
      const int64_t key = j < run_len ? runs[0] + j : runs[2] + (j - run_len);
      const int64_t slot = oracle_cache_offset(cache, layer, kv_head, key);
      key_rows[j] = cache->keys + slot;
      value_rows[j] = cache->values + slot;
    }
    scores.resize(std::max<int64_t>(keys, 1));
    oracle_attend(qkv + row * stride + head * d, (int)d, (int)keys, key_rows.data(),
                  value_rows.data(), scores.data(), out + row * width + head * d);
  }
}

}  // namespace

extern "C" {

void oracle_rope_inv_freq(float base, int head_dim, float* out) {
  for (int i = 0; i < head_dim / 2; ++i) {
    out[i] = 1.0f / std::pow(base, (float)(2 * i) / (float)head_dim);
  }
}

void oracle_rope_half(float* head, int head_dim, const float* cos, const float* sin) {
  const int half = head_dim / 2;
  for (int i = 0; i < half; ++i) {
    const float x = head[i], y = head[i + half];
    head[i] = x * cos[i] - y * sin[i];
    head[i + half] = y * cos[i] + x * sin[i];
  }
}

void oracle_rope_interleaved(float* head, int head_dim, const float* cos, const float* sin) {
  for (int i = 0; i < head_dim / 2; ++i) {
    const float x = head[2 * i], y = head[2 * i + 1];
    head[2 * i] = x * cos[i] - y * sin[i];
    head[2 * i + 1] = y * cos[i] + x * sin[i];
  }
}

int oracle_rotary_angles(int kind, const int64_t* params, float base, int head_dim,
                         float spatial_scale, const int64_t* position, float* cos, float* sin) {
  const int half = head_dim / 2;
  std::vector<float> inv_freq(half, 0.0f);
  std::vector<int> axes(half, 0);  // 0 temporal, 1 height, 2 width
  auto sections_axes = [&](const int64_t* sections) {
    if (sections[0] + sections[1] + sections[2] != half) return false;
    int at = 0;
    for (int axis = 0; axis < 3; ++axis)
      for (int64_t i = 0; i < sections[axis]; ++i) axes[at++] = axis;
    return true;
  };
  switch (kind) {
    case ORACLE_ROT_SEQUENCE:
      oracle_rope_inv_freq(base, head_dim, inv_freq.data());
      break;
    case ORACLE_ROT_LINEAR:
      oracle_rope_inv_freq(base, head_dim, inv_freq.data());
      for (auto& f : inv_freq) f = f / (float)params[0];
      break;
    case ORACLE_ROT_PARTIAL:
      oracle_rope_inv_freq(base, head_dim, inv_freq.data());
      for (int i = (int)params[0]; i < half; ++i) inv_freq[i] = 0.0f;
      break;
    case ORACLE_ROT_MULTIMODAL:
      oracle_rope_inv_freq(base, head_dim, inv_freq.data());
      if (!sections_axes(params)) return -1;
      break;
    case ORACLE_ROT_AXES:
    case ORACLE_ROT_GRID: {
      int64_t grid[3] = {0, half / 2, half / 2};
      const int64_t* sections = kind == ORACLE_ROT_GRID ? grid : params;
      int at = 0;
      for (int axis = 0; axis < 3; ++axis) {
        std::vector<float> part(sections[axis]);
        oracle_rope_inv_freq(base, (int)(2 * sections[axis]), part.data());
        for (int64_t i = 0; i < sections[axis] && at < half; ++i) inv_freq[at++] = part[i];
      }
      if (!sections_axes(sections)) return -1;
      break;
    }
    case ORACLE_ROT_MULTIMODAL_INTERLEAVED:
      oracle_rope_inv_freq(base, head_dim, inv_freq.data());
      for (int i = 0; i < half; ++i) {
        const int m = i % 3;
        axes[i] = (m == 1 && i < 3 * params[1]) ? 1 : (m == 2 && i < 3 * params[2]) ? 2 : 0;
      }
      break;
    default:
      return -1;
  }
  for (int i = 0; i < half; ++i) {
    float frequency = inv_freq[i];
    if (axes[i] != 0) frequency = frequency * spatial_scale;
    const float angle = (float)position[axes[i]] * frequency;
    cos[i] = std::cos(angle);
    sin[i] = std::sin(angle);
  }
  return 0;
}

float oracle_exp(float x) {
  x = clampf(x, kExpMin, kExpMax);
  const float exponent = round_even(x * kLog2E);
  const float remainder = x - exponent * kLn2High - exponent * kLn2Low;
  float poly = kExpPoly[0];
  for (int i = 1; i < 6; ++i) poly = poly * remainder + kExpPoly[i];
  poly = poly * remainder * remainder + remainder + 1.0f;
  return poly * from_bits((uint32_t)(((int32_t)exponent + kExpBias) << 23));
}

float oracle_exp_fast(float x) {
  x = maxf(x, kExpMin);
  const float exponent = round_even(x * kLog2E);
  const float remainder = std::fma(-exponent, kLn2, x);
  float poly = kExpTaylor[0];
  for (int i = 1; i < 5; ++i) poly = std::fma(poly, remainder, kExpTaylor[i]);
  return poly * from_bits((uint32_t)(((int32_t)exponent + kExpBias) << 23));
}

float oracle_round_bf16(float value) {
  const uint32_t bits = to_bits(value);
  const uint32_t rounding = 0x7FFFu + ((bits >> 16) & 1u);
  return from_bits((bits + rounding) & 0xFFFF0000u);
}

float oracle_exponentials_apply(int fast, float* scores, int n) {
  float max = -INFINITY;
  for (int i = 0; i < n; ++i) max = maxf(max, scores[i]);
  float (*exponential)(float) = fast ? oracle_exp_fast : oracle_exp;
  float sums[kExpRun];
  for (int i = 0; i < kExpRun; ++i) sums[i] = 0.0f;
  const int whole = n / kExpRun * kExpRun;
  for (int i = 0; i < whole; ++i) {
    scores[i] = exponential(scores[i] - max);
    sums[i % kExpRun] += scores[i];
  }
  for (int i = whole; i < n; ++i) scores[i] = exponential(scores[i] - max);
  // `rest.iter().chain(&sums).sum()`: the tail first, then the run sums, from -0.0.
  float total = -0.0f;
  for (int i = whole; i < n; ++i) total += scores[i];
  for (int i = 0; i < kExpRun; ++i) total += sums[i];
  return total;
}

void oracle_softmax(float* scores, int n) {
  float max = -INFINITY;
  for (int i = 0; i < n; ++i) max = maxf(max, scores[i]);
  for (int i = 0; i < n; ++i) scores[i] = oracle_exp(scores[i] - max);
  float total = -0.0f;
  for (int i = 0; i < n; ++i) total += scores[i];
  for (int i = 0; i < n; ++i) scores[i] /= total;
}

float oracle_dot(const float* left, const float* right, int n) {
  float sum = -0.0f;
  for (int i = 0; i < n; ++i) sum += left[i] * right[i];
  return sum;
}

void oracle_rms_norm(const float* x, const float* weight, float eps, int dim, float* out) {
  const float mean = oracle_dot(x, x, dim) / (float)dim;
  const float inverse = 1.0f / std::sqrt(mean + eps);
  for (int i = 0; i < dim; ++i) out[i] = x[i] * inverse * weight[i];
}

void oracle_attend(const float* query, int head_dim, int keys, const float* const* key_rows,
                   const float* const* value_rows, float* scores, float* out) {
  const float scale = 1.0f / std::sqrt((float)head_dim);
  for (int j = 0; j < keys; ++j) scores[j] = oracle_dot(query, key_rows[j], head_dim) * scale;
  // weigh (ops.rs:329-342): the DOTS=4 blocks of axpy_f32_many add each row's product on its
  // own, in key order -- the same arithmetic as one key at a time.
  oracle_softmax(scores, keys);
  for (int i = 0; i < head_dim; ++i) out[i] = 0.0f;
  for (int j = 0; j < keys; ++j) {
    const float weight = scores[j];
    const float* value = value_rows[j];
    for (int i = 0; i < head_dim; ++i) out[i] += weight * value[i];
  }
}

void oracle_mask_keys(const oracle_mask* mask, int64_t position, int64_t end, int64_t* runs) {
  runs[2] = runs[3] = 0;
  switch (mask->kind) {
    case ORACLE_MASK_CAUSAL:
      runs[0] = 0;
      runs[1] = position + 1;
      return;
    case ORACLE_MASK_WINDOW:
      runs[0] = std::max<int64_t>(position + 1 - mask->window, 0);
      runs[1] = position + 1;
      return;
    case ORACLE_MASK_FULL:
      runs[0] = 0;
      runs[1] = end;
      return;
    case ORACLE_MASK_GROUPS: {
      if (position < mask->state) {
        runs[0] = 0;
        runs[1] = end;
        return;
      }
      // partition_point(|&e| e <= position)
      int64_t group = 0;
      while (group < mask->n_ends && mask->ends[group] <= position) ++group;
      const int64_t start = group == 0 ? mask->state : mask->ends[group - 1];
      runs[0] = 0;
      runs[1] = mask->state;
      runs[2] = start;
      runs[3] = mask->ends[group];
      return;
    }
    default:
      runs[0] = runs[1] = 0;
  }
}

int64_t oracle_cache_offset(const oracle_cache* cache, int64_t layer, int64_t kv_head,
                            int64_t position) {
  const int64_t slot = position % cache->capacity;
  return ((layer * cache->kv_heads + kv_head) * cache->capacity + slot) * cache->head_dim;
}

void oracle_cache_keep(oracle_cache* cache, int64_t layer, int64_t unit, int64_t position,
                       const float* head) {
  if (unit < cache->heads) return;
  float* target = unit < cache->heads + cache->kv_heads ? cache->keys : cache->values;
  const int64_t at =
      oracle_cache_offset(cache, layer, (unit - cache->heads) % cache->kv_heads, position);
  std::memcpy(target + at, head, sizeof(float) * cache->head_dim);
}

int oracle_span_fits(const oracle_cache* cache, int64_t rows, int64_t first,
                     const oracle_mask* mask) {
  const int64_t reach = mask->kind == ORACLE_MASK_WINDOW ? mask->window + rows : first + rows;
  return reach <= cache->capacity ? 1 : 0;
}

void oracle_attention_input(oracle_cache* cache, int64_t layer, int64_t rows, int64_t first,
                            int rope, const float* angles, const float* q_norm,
                            const float* k_norm, float norm_eps, float* qkv, int64_t stride) {
  const int64_t d = cache->head_dim;
  const int64_t units = cache->heads + 2 * cache->kv_heads;
  const int64_t rotated = cache->heads + cache->kv_heads;
  std::vector<float> copy(d);
  for (int64_t row = 0; row < rows; ++row) {
    const int64_t position = first + row;
    const float* cos = angles ? angles + row * d : nullptr;
    const float* sin = angles ? cos + d / 2 : nullptr;
    for (int64_t unit = 0; unit < units; ++unit) {
      float* head = qkv + row * stride + unit * d;
      if (unit < rotated) {
        const float* weight = unit < cache->heads ? q_norm : k_norm;
        if (weight != nullptr) {
          std::memcpy(copy.data(), head, sizeof(float) * d);
          oracle_rms_norm(copy.data(), weight, norm_eps, (int)d, head);
        }
        if (rope == 1) oracle_rope_half(head, (int)d, cos, sin);
        if (rope == 2) oracle_rope_interleaved(head, (int)d, cos, sin);
      }
      oracle_cache_keep(cache, layer, unit, position, head);
    }
  }
}

void oracle_cache_attend(const oracle_cache* cache, int64_t layer, int64_t rows, int64_t first,
                         const oracle_mask* mask, const float* qkv, int64_t stride, float* out) {
  std::vector<float> scores;
  std::vector<const float*> key_rows, value_rows;
  for (int64_t head = 0; head < cache->heads; ++head)
    attend_head(cache, layer, rows, first, mask, qkv, stride, out, head, scores, key_rows,
                value_rows);
}

void oracle_cache_attend_team(const oracle_cache* cache, int64_t layer, int64_t rows,
                              int64_t first, const oracle_mask* mask, const float* qkv,
                              int64_t stride, float* out, int threads) {
  std::function<void(int, int)> task = [&](int index, int count) {
    std::vector<float> scores;
    std::vector<const float*> key_rows, value_rows;
    auto share = Team::split(cache->heads, 1, index, count);
    for (int64_t head = share.first; head < share.second; ++head)
      attend_head(cache, layer, rows, first, mask, qkv, stride, out, head, scores, key_rows,
                  value_rows);
  };
  team(threads).run(task);
}

void oracle_decode_batch_team(const oracle_cache* caches, int64_t batch, int64_t layer,
                              const int64_t* firsts, const float* qkv, int64_t stride,
                              float* out, int64_t out_stride, int threads) {
  oracle_mask causal{ORACLE_MASK_CAUSAL, 0, 0, nullptr, 0};
  for (int64_t s = 0; s < batch; ++s) {
    oracle_cache_attend_team(&caches[s], layer, 1, firsts[s], &causal, qkv + s * stride, stride,
                             out + s * out_stride, threads);
  }
}

void oracle_attend_call(int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t images,
                        int64_t queries, int64_t keys, const float* q, int64_t q_stride,
                        int64_t q_offset, const float* k, int64_t k_stride, int64_t k_offset,
                        const float* v, int64_t v_stride, int64_t v_offset, float* out,
                        int64_t head_begin, int64_t head_end, int64_t query_begin,
                        int64_t query_end, int threads) {
  const int64_t group = heads / kv_heads;
  const int64_t sampled_heads = head_end - head_begin;
  const int64_t units = images * sampled_heads;
  std::function<void(int, int)> task = [&](int index, int count) {
    std::vector<float> scores(std::max<int64_t>(keys, 1));
    std::vector<const float*> key_rows(keys), value_rows(keys);
    // Split (image, head, query) units so that a sample of few heads still spreads over the
    // team, as the reference splits (image, head, query block) units (attention.rs:81-95).
    const int64_t total = units * (query_end - query_begin);
    auto share = Team::split(total, 1, index, count);
    int64_t cached_unit = -1;
    for (int64_t u = share.first; u < share.second; ++u) {
      const int64_t unit = u / (query_end - query_begin);
      const int64_t query = query_begin + u % (query_end - query_begin);
      const int64_t image = unit / sampled_heads, head = head_begin + unit % sampled_heads;
      const int64_t kv_head = head / group;
      if (unit != cached_unit) {
        for (int64_t j = 0; j < keys; ++j) {
          key_rows[j] = k + (image * keys + j) * k_stride + k_offset + kv_head * head_dim;
          value_rows[j] = v + (image * keys + j) * v_stride + v_offset + kv_head * head_dim;
        }
        cached_unit = unit;
      }
      const int64_t row = image * queries + query;
      oracle_attend(q + row * q_stride + q_offset + head * head_dim, (int)head_dim, (int)keys,
                    key_rows.data(), value_rows.data(), scores.data(),
                    out + row * heads * head_dim + head * head_dim);
    }
  };
  team(std::max(threads, 1)).run(task);
}

void oracle_qk_prologue(int64_t tokens, int64_t heads, int64_t head_dim, int norm, int rope,
                        int64_t rotated, const float* angles, const float* q_norm,
                        const float* k_norm, float eps, float* qkv, int64_t stride) {
  const int64_t d = head_dim, width = heads * d;
  std::vector<float> scratch(width);
  for (int64_t t = 0; t < tokens; ++t) {
    for (int part = 0; part < 2; ++part) {
      float* run = qkv + t * stride + part * width;
      const float* weight = part == 0 ? q_norm : k_norm;
      if (norm == 1) {
        // rms_rows: rms_norm of the run into scratch, copied back
        oracle_rms_norm(run, weight, eps, (int)width, scratch.data());
        std::memcpy(run, scratch.data(), sizeof(float) * width);
      } else if (norm == 2) {
        // normalize_heads: rms_norm's rows of weight.len() = head_dim
        for (int64_t h = 0; h < heads; ++h)
          oracle_rms_norm(run + h * d, weight, eps, (int)d, scratch.data() + h * d);
        std::memcpy(run, scratch.data(), sizeof(float) * width);
      }
    }
  }
  if (rope == 0) return;
  for (int64_t t = 0; t < tokens && t < rotated; ++t) {
    const float* cos = angles + t * d;
    const float* sin = cos + d / 2;
    // the queries and keys of the token, head_dim chunks of its first 2 * width values
    for (int64_t h = 0; h < 2 * heads; ++h) {
      float* head = qkv + t * stride + h * d;
      if (rope == 1) oracle_rope_half(head, (int)d, cos, sin);
      else oracle_rope_interleaved(head, (int)d, cos, sin);
    }
  }
}

static float oracle_sigmoid(float x) { return 1.0f / (1.0f + oracle_exp(-x)); }

void oracle_gated_input(oracle_cache* cache, int64_t layer, int64_t rows, int64_t first, int gate,
                        int64_t rotary_dim, const float* angles, const float* q_norm,
                        const float* k_norm, float norm_eps, float* qkv, int64_t stride) {
  const int64_t d = cache->head_dim, heads = cache->heads, kv = cache->kv_heads;
  const int64_t gate_heads = gate == 1 ? heads : 0;
  const int64_t units = heads + gate_heads + 2 * kv;
  std::vector<float> copy(d);
  for (int64_t row = 0; row < rows; ++row) {
    const int64_t position = first + row;
    const float* cos = angles + row * rotary_dim;
    const float* sin = cos + rotary_dim / 2;
    for (int64_t unit = 0; unit < units; ++unit) {
      float* head = qkv + row * stride + unit * d;
      if (unit >= heads && unit < heads + gate_heads) {  // Role::Gate
        for (int64_t e = 0; e < d; ++e) head[e] = oracle_sigmoid(head[e]);
        continue;
      }
      const int64_t cache_unit = unit - gate_heads;  // Role::Key / Role::Value numbering
      if (cache_unit < heads + kv) {                 // Role::Query or Role::Key: position()
        const float* weight = cache_unit < heads ? q_norm : k_norm;
        if (weight != nullptr) {
          std::memcpy(copy.data(), head, sizeof(float) * d);
          oracle_rms_norm(copy.data(), weight, norm_eps, (int)d, head);
        }
        oracle_rope_half(head, (int)rotary_dim, cos, sin);
      }
      if (cache_unit >= heads) oracle_cache_keep(cache, layer, cache_unit, position, head);
    }
    if (gate == 2) {  // project_head_gates
      float* gates = qkv + row * stride + units * d;
      for (int64_t h = 0; h < heads; ++h) gates[h] = oracle_sigmoid(gates[h]);
    }
  }
}

void oracle_gate(int64_t rows, int64_t heads, int64_t kv_heads, int64_t head_dim, int gate,
                 const float* qkv, int64_t stride, float* attention) {
  if (gate == 0) return;
  const int64_t d = head_dim, width = heads * d;
  const int64_t head_columns = (heads + (gate == 1 ? heads : 0) + 2 * kv_heads) * d;
  for (int64_t h = 0; h < heads; ++h) {
    for (int64_t row = 0; row < rows; ++row) {
      const float* r = qkv + row * stride;
      float* attended = attention + row * width + h * d;
      for (int64_t e = 0; e < d; ++e)
        attended[e] *= gate == 1 ? r[(heads + h) * d + e] : r[head_columns + h];
    }
  }
}

/* One block of 32 values as Q7b32 levels (quant.rs:142-149): returns the scale. */
static float oracle_q7_block(const float* x, int8_t* levels) {
  float absmax = 0.0f;
  for (int i = 0; i < 32; ++i) absmax = maxf(absmax, std::fabs(x[i]));
  const float scale = absmax == 0.0f ? 1.0f : absmax / 63.0f;
  for (int i = 0; i < 32; ++i) {
    float l = std::nearbyint(x[i] / scale);  // ties to even (the default rounding mode)
    if (l > 63.0f) l = 63.0f;
    if (l < -63.0f) l = -63.0f;
    levels[i] = (int8_t)l;
  }
  return scale;
}

/* One block of 32 activations as int8 (d = absmax / 127, ties-even). */
static float oracle_a8_block(const float* x, int8_t* levels) {
  float absmax = 0.0f;
  for (int i = 0; i < 32; ++i) absmax = maxf(absmax, std::fabs(x[i]));
  const float scale = absmax == 0.0f ? 1.0f : absmax / 127.0f;
  for (int i = 0; i < 32; ++i) {
    float l = std::nearbyint(x[i] / scale);
    if (l > 127.0f) l = 127.0f;
    if (l < -127.0f) l = -127.0f;
    levels[i] = (int8_t)l;
  }
  return scale;
}

void oracle_attend_int8(int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t queries,
                        int64_t keys, const float* q, int64_t q_stride, const float* k,
                        int64_t k_stride, const float* v, int64_t v_stride, int fast, float* out) {
  const int64_t d = head_dim, dp = (d + 31) / 32 * 32, kp = (keys + 31) / 32 * 32;
  const int64_t db = dp / 32, kb = kp / 32;
  std::vector<float> mean(d), row(std::max(dp, kp)), scores(keys);
  std::vector<int8_t> kq(keys * dp), vq(d * kp), aq(std::max(dp, kp));
  std::vector<float> ks(keys * db), vs(d * kb), as_(std::max(db, kb));
  const int64_t group = heads / kv_heads;
  for (int64_t kvh = 0; kvh < kv_heads; ++kvh) {
    // the keys less their mean, as Q7b32 rows of dp values
    for (int64_t e = 0; e < d; ++e) mean[e] = 0.0f;
    for (int64_t j = 0; j < keys; ++j)
      for (int64_t e = 0; e < d; ++e) mean[e] += k[j * k_stride + kvh * d + e];
    for (int64_t e = 0; e < d; ++e) mean[e] /= (float)keys;
    for (int64_t j = 0; j < keys; ++j) {
      for (int64_t e = 0; e < dp; ++e) row[e] = e < d ? k[j * k_stride + kvh * d + e] - mean[e] : 0.0f;
      for (int64_t b = 0; b < db; ++b) ks[j * db + b] = oracle_q7_block(&row[b * 32], &kq[j * dp + b * 32]);
    }
    // the values transposed: a row per channel over kp keys
    for (int64_t e = 0; e < d; ++e) {
      for (int64_t j = 0; j < kp; ++j) row[j] = j < keys ? v[j * v_stride + kvh * d + e] : 0.0f;
      for (int64_t b = 0; b < kb; ++b) vs[e * kb + b] = oracle_q7_block(&row[b * 32], &vq[e * kp + b * 32]);
    }
    for (int64_t hh = 0; hh < group; ++hh) {
      const int64_t h = kvh * group + hh;
      for (int64_t i = 0; i < queries; ++i) {
        for (int64_t e = 0; e < dp; ++e) row[e] = e < d ? q[i * q_stride + h * d + e] : 0.0f;
        for (int64_t b = 0; b < db; ++b) as_[b] = oracle_a8_block(&row[b * 32], &aq[b * 32]);
        const float scale = 1.0f / std::sqrt((float)d);
        for (int64_t j = 0; j < keys; ++j) {
          float s = 0.0f;
          for (int64_t b = 0; b < db; ++b) {
            int32_t acc = 0;
            for (int t = 0; t < 32; ++t) acc += int32_t(kq[j * dp + b * 32 + t]) * int32_t(aq[b * 32 + t]);
            s += (float)acc * (ks[j * db + b] * as_[b]);
          }
          scores[j] = s * scale;
        }
        const float sum = oracle_exponentials_apply(fast, scores.data(), (int)keys);
        // the exponentials as int8 activations of P.V^T
        for (int64_t j = 0; j < kp; ++j) row[j] = j < keys ? scores[j] : 0.0f;
        for (int64_t b = 0; b < kb; ++b) as_[b] = oracle_a8_block(&row[b * 32], &aq[b * 32]);
        for (int64_t e = 0; e < d; ++e) {
          float o = 0.0f;
          for (int64_t b = 0; b < kb; ++b) {
            int32_t acc = 0;
            for (int t = 0; t < 32; ++t) acc += int32_t(vq[e * kp + b * 32 + t]) * int32_t(aq[b * 32 + t]);
            o += (float)acc * (vs[e * kb + b] * as_[b]);
          }
          out[i * heads * d + h * d + e] = o / sum;
        }
      }
    }
  }
}

void oracle_relpos_attend(int64_t heads, int64_t head_dim, int64_t frames, const float* q,
                          const float* k, const float* v, int64_t qkv_stride,
                          const float* positions, int64_t positions_stride, const float* bias_u,
                          const float* bias_v, float* out) {
  const int64_t d = head_dim;
  std::vector<float> content(d), position(d), scores(frames);
  const float scale = 1.0f / std::sqrt((float)d);
  for (int64_t h = 0; h < heads; ++h) {
    for (int64_t i = 0; i < frames; ++i) {
      // biased_queries (attention.rs:77-99): f32 sums
      const float* query = q + i * qkv_stride + h * d;
      for (int64_t e = 0; e < d; ++e) {
        content[e] = query[e] + bias_u[h * d + e];
        position[e] = query[e] + bias_v[h * d + e];
      }
      // scores (attention.rs:101-135): the content dot, plus the position dot, then the scale
      for (int64_t j = 0; j < frames; ++j) {
        const float c = oracle_dot(k + j * qkv_stride + h * d, content.data(), (int)d);
        const float* r = positions + (frames - 1 - i + j) * positions_stride + h * d;
        float s = c;
        s += oracle_dot(r, position.data(), (int)d);
        scores[j] = s * scale;
      }
      // mix (attention.rs:137-159): softmax, then the values key by key
      oracle_softmax(scores.data(), (int)frames);
      float* o = out + i * heads * d + h * d;
      for (int64_t e = 0; e < d; ++e) o[e] = 0.0f;
      for (int64_t j = 0; j < frames; ++j) {
        const float* value = v + j * qkv_stride + h * d;
        for (int64_t e = 0; e < d; ++e) o[e] += scores[j] * value[e];
      }
    }
  }
}

void oracle_team_release(void) {
  delete current_team;
  current_team = nullptr;
}

void oracle_reference_attend_f64(const double* qkv_heads, int64_t rows, int64_t heads,
                                 int64_t kv_heads, int64_t head_dim, const oracle_mask* mask,
                                 double* out) {
  const int64_t units = heads + 2 * kv_heads;
  const int64_t group = heads / kv_heads;
  auto head_at = [&](int64_t row, int64_t unit) { return qkv_heads + (row * units + unit) * head_dim; };
  std::vector<int64_t> seen;
  std::vector<double> scores;
  for (int64_t row = 0; row < rows; ++row) {
    seen.clear();
    switch (mask->kind) {
      case ORACLE_MASK_CAUSAL:
        for (int64_t j = 0; j <= row; ++j) seen.push_back(j);
        break;
      case ORACLE_MASK_WINDOW:
        for (int64_t j = std::max<int64_t>(row + 1 - mask->window, 0); j <= row; ++j)
          seen.push_back(j);
        break;
      case ORACLE_MASK_GROUPS:
        if (row >= mask->state) {
          int64_t end = -1, start = mask->state;
          for (int64_t g = 0; g < mask->n_ends; ++g)
            if (mask->ends[g] > row) { end = mask->ends[g]; break; }
          for (int64_t g = mask->n_ends - 1; g >= 0; --g)
            if (mask->ends[g] <= row) { start = mask->ends[g]; break; }
          for (int64_t j = 0; j < mask->state; ++j) seen.push_back(j);
          for (int64_t j = start; j < end; ++j) seen.push_back(j);
          break;
        }
        for (int64_t j = 0; j < rows; ++j) seen.push_back(j);
        break;
      case 4:  // Prefix(count)
        if (row < mask->window) {
          for (int64_t j = 0; j < mask->window; ++j) seen.push_back(j);
        } else {
          for (int64_t j = 0; j < mask->window; ++j) seen.push_back(j);
          seen.push_back(row);
        }
        break;
      default:  // Full
        for (int64_t j = 0; j < rows; ++j) seen.push_back(j);
    }
    for (int64_t head = 0; head < heads; ++head) {
      const double* query = head_at(row, head);
      scores.assign(seen.size(), 0.0);
      double max = -INFINITY;
      for (size_t s = 0; s < seen.size(); ++s) {
        const double* key = head_at(seen[s], heads + head / group);
        double dot = 0.0;
        for (int64_t i = 0; i < head_dim; ++i) dot += query[i] * key[i];
        scores[s] = dot / std::sqrt((double)head_dim);
        max = std::max(max, scores[s]);
      }
      double total = 0.0;
      for (auto& score : scores) {
        score = std::exp(score - max);
        total += score;
      }
      double* mixed = out + (row * heads + head) * head_dim;
      for (int64_t i = 0; i < head_dim; ++i) mixed[i] = 0.0;
      for (size_t s = 0; s < seen.size(); ++s) {
        const double* value = head_at(seen[s], heads + kv_heads + head / group);
        for (int64_t i = 0; i < head_dim; ++i) mixed[i] += scores[s] / total * value[i];
      }
    }
  }
}

}  // extern "C"
