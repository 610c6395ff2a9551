// oracle.cpp -- TEST INFRASTRUCTURE ONLY (see oracle.h for scope and pins).
//
// Every function restates one reference function, cited as file:line relative
// to the reference project root. Compile with -ffp-contract=off and without
// -ffast-math: each `a * b + c` below must round twice, as Rust (which never
// contracts) does, and every Rust `mul_add` is written as fmaf.

#include "oracle.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <functional>
#include <limits>
#include <mutex>
#include <thread>
#include <vector>

namespace {

// ---------------------------------------------------------------------------
// A small persistent thread pool that restates the reference's rayon splits:
// a parallel loop over `tasks` independent items, dealt out dynamically.
// ---------------------------------------------------------------------------
class Pool {
 public:
  static Pool& get() {
    static Pool pool;
    return pool;
  }

  void set_threads(int n) {
    std::lock_guard<std::mutex> lock(config_mutex_);
    stop_workers();
    threads_ = std::max(1, n);
    start_workers();
  }
  int threads() const { return threads_; }

  // Runs fn(i) for i in [0, tasks), splitting the range over the workers.
  void parallel_for(int64_t tasks, const std::function<void(int64_t, int64_t)>& fn) {
    if (tasks <= 0) return;
    if (threads_ <= 1 || tasks == 1) {
      fn(0, tasks);
      return;
    }
    std::lock_guard<std::mutex> lock(config_mutex_);
    const int64_t grain = std::max<int64_t>(1, tasks / (int64_t(threads_) * 16));
    {
      std::lock_guard<std::mutex> g(mutex_);
      job_ = &fn;
      job_tasks_ = tasks;
      job_grain_ = grain;
      next_.store(0);
      pending_ = threads_ - 1;
      ++generation_;
    }
    cv_.notify_all();
    run_share();
    std::unique_lock<std::mutex> g(mutex_);
    done_cv_.wait(g, [&] { return pending_ == 0; });
    job_ = nullptr;
  }

 private:
  Pool() {
    unsigned hw = std::thread::hardware_concurrency();
    threads_ = hw == 0 ? 1 : int(hw);
    start_workers();
  }
  ~Pool() { stop_workers(); }

  void run_share() {
    for (;;) {
      const int64_t begin = next_.fetch_add(job_grain_);
      if (begin >= job_tasks_) break;
      (*job_)(begin, std::min(job_tasks_, begin + job_grain_));
    }
  }

  // `seen` is the generation current when the worker was created (read under
  // the lock by start_workers), so a job posted before this thread first runs
  // is still picked up.
  void worker(uint64_t seen) {
    for (;;) {
      {
        std::unique_lock<std::mutex> g(mutex_);
        cv_.wait(g, [&] { return quit_ || generation_ != seen; });
        if (quit_) return;
        seen = generation_;
      }
      run_share();
      std::lock_guard<std::mutex> g(mutex_);
      if (--pending_ == 0) done_cv_.notify_one();
    }
  }

  void start_workers() {
    uint64_t current;
    {
      std::lock_guard<std::mutex> g(mutex_);
      quit_ = false;
      current = generation_;
    }
    for (int i = 1; i < threads_; ++i)
      workers_.emplace_back([this, current] { worker(current); });
  }
  void stop_workers() {
    {
      std::lock_guard<std::mutex> g(mutex_);
      quit_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
    workers_.clear();
  }

  int threads_ = 1;
  std::vector<std::thread> workers_;
  std::mutex config_mutex_;
  std::mutex mutex_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(int64_t, int64_t)>* job_ = nullptr;
  int64_t job_tasks_ = 0, job_grain_ = 1;
  std::atomic<int64_t> next_{0};
  int pending_ = 0;
  uint64_t generation_ = 0;
  bool quit_ = false;
};

void parallel_for(int64_t tasks, const std::function<void(int64_t, int64_t)>& fn) {
  Pool::get().parallel_for(tasks, fn);
}

// cpu-kernels/src/lib.rs:16 -- PARALLEL_THRESHOLD.
constexpr int64_t kParallelThreshold = int64_t(1) << 18;

// Rust `f32 as i32`: saturating, NaN -> 0.
int32_t rust_f32_as_i32(float v) {
  if (std::isnan(v)) return 0;
  if (v >= 2147483647.0f) return std::numeric_limits<int32_t>::max();
  if (v <= -2147483648.0f) return std::numeric_limits<int32_t>::min();
  return int32_t(v);
}

// Rust `f32::powi` lowers to the compiler builtin __powisf2 (repeated
// squaring, reciprocal for a negative exponent); restated literally so that
// overflow of 2^|i| to +inf (and hence 2^i -> 0) behaves the same.
float rust_powi_f32(float a, int32_t b) {
  const bool recip = b < 0;
  float r = 1.0f;
  for (;;) {
    if (b & 1) r *= a;
    b /= 2;
    if (b == 0) break;
    a *= a;
  }
  return recip ? 1.0f / r : r;
}

template <typename T>
void rope_impl(const T* x, T* y, const T* cos_t, const T* sin_t, int64_t n_vec, int64_t seq,
               int64_t batch, int64_t head_dim, int64_t rotary_dim, int64_t s_vec,
               int64_t s_pos, int64_t s_batch, int64_t s_feat) {
  const int64_t half = rotary_dim / 2;
  parallel_for(batch * seq, [&](int64_t t0, int64_t t1) {
    for (int64_t t = t0; t < t1; ++t) {
      const int64_t b = t / seq, p = t % seq;
      for (int64_t v = 0; v < n_vec; ++v) {
        const int64_t base = v * s_vec + p * s_pos + b * s_batch;
        for (int64_t i = 0; i < half; ++i) {
          const T c = cos_t[p * half + i], s = sin_t[p * half + i];
          const T x1 = x[base + i * s_feat], x2 = x[base + (i + half) * s_feat];
          const T a = x1 * c;
          const T bb = x2 * s;
          const T cc = x1 * s;
          const T dd = x2 * c;
          y[base + i * s_feat] = a - bb;
          y[base + (i + half) * s_feat] = cc + dd;
        }
        for (int64_t j = rotary_dim; j < head_dim; ++j)
          y[base + j * s_feat] = x[base + j * s_feat];
      }
    }
  });
}

}  // namespace

extern "C" {

void orc_set_threads(int threads) { Pool::get().set_threads(threads); }
int orc_threads(void) { return Pool::get().threads(); }

// ---------------------------------------------------------------------------
// crates/cpu-kernels/src/lib.rs:474-505 -- mlx_expm1f.
// ---------------------------------------------------------------------------
float orc_expm1_mlx_f32(float a) {
  float j = fmaf(1.442695f, a, 12582912.0f);
  j -= 12582912.0f;
  const int32_t i = rust_f32_as_i32(j);
  const float f = fmaf(j, -0.693145752f, a);
  const float s = (a == 0.0f) ? a : f * f;
  float r = 1.9735098e-4f;
  r = fmaf(r, f, 1.3930907e-3f);
  r = fmaf(r, f, 8.33344e-3f);
  r = fmaf(r, f, 4.1666802e-2f);
  r = fmaf(r, f, 1.6666672e-1f);
  r = fmaf(r, f, 4.9999997e-1f);
  const float u = (j == 1.0f) ? f + 0.5f : f;
  const float v = fmaf(r, s, u);
  const float half = 0.5f;
  const float t = half * rust_powi_f32(2.0f, i);
  const float y = t - half;
  const float x = (t - y) - half;
  r = fmaf(v, t, x) + y;
  r += r;
  if (j == 0.0f) r = v;
  if (j == 1.0f) r = v + v;
  if (std::fabs(a - 1.0f) > 88.0f) {
    const float e = exp2f(a);
    r = fmaf(e, e, -1.0f);
  }
  return r;
}

// ---------------------------------------------------------------------------
// crates/cpu-kernels/src/lib.rs:449-471 -- erf_f32 (MLX Metal erff sequence).
// ---------------------------------------------------------------------------
float orc_erf_f32(float a) {
  const float t = std::fabs(a);
  const float s = a * a;
  if (t > 0.9277344f) {
    float r = fmaf(-1.7285347e-5f, t, 3.8319713e-4f);
    const float u = fmaf(-3.8839644e-3f, t, 2.4254622e-2f);
    r = fmaf(r, s, u);
    r = fmaf(r, t, -1.0677788e-1f);
    r = fmaf(r, t, -6.3484669e-1f);
    r = fmaf(r, t, -1.2871751e-1f);
    r = fmaf(r, t, -t);
    r = -orc_expm1_mlx_f32(r);
    return std::copysign(r, a);
  }
  float r = -5.967617e-4f;
  r = fmaf(r, s, 4.9911942e-3f);
  r = fmaf(r, s, -2.6768135e-2f);
  r = fmaf(r, s, 1.1281992e-1f);
  r = fmaf(r, s, -3.7612534e-1f);
  r = fmaf(r, s, 1.2837917e-1f);
  return fmaf(r, a, a);
}

// crates/cpu-kernels/src/lib.rs:509-511 -- 0.5 * x * (1 + erf(x * FRAC_1_SQRT_2)),
// evaluated left to right: (0.5 * x) * (1 + erf(...)).
float orc_gelu_erf_f32(float x) {
  return 0.5f * x * (1.0f + orc_erf_f32(x * 0.70710678118654752440f));
}

// ErfOp over a tensor (tenferro-ext/src/lib.rs:132-170): elementwise erf_f32.
void orc_erf_f32_n(const float* x, float* y, int64_t n) {
  parallel_for((n + 4095) / 4096, [&](int64_t c0, int64_t c1) {
    for (int64_t i = c0 * 4096; i < std::min(n, c1 * 4096); ++i) y[i] = orc_erf_f32(x[i]);
  });
}

void orc_gelu_erf_f32_n(const float* x, float* y, int64_t n) {
  parallel_for((n + 4095) / 4096, [&](int64_t c0, int64_t c1) {
    for (int64_t i = c0 * 4096; i < std::min(n, c1 * 4096); ++i) y[i] = orc_gelu_erf_f32(x[i]);
  });
}

// ---------------------------------------------------------------------------
// crates/cpu-kernels/src/lib.rs:397-443 -- layer_norm_feature_first_into.
// Column c is the contiguous slice [c*d, (c+1)*d). Three sequential passes:
// sum, centered sum of squares, write.
// ---------------------------------------------------------------------------
void orc_layer_norm_feature_first_f32(const float* x, int64_t d, int64_t cols,
                                      const float* weight, const float* bias, float eps,
                                      float* y) {
  if (d == 0 || cols == 0) return;
  const float denom = float(d);
  auto normalize = [&](float* out, const float* input) {
    float mean = 0.0f;
    for (int64_t i = 0; i < d; ++i) mean += input[i];
    mean /= denom;
    float var = 0.0f;
    for (int64_t i = 0; i < d; ++i) {
      const float centered = input[i] - mean;
      var += centered * centered;
    }
    var /= denom;
    const float inv = 1.0f / std::sqrt(var + eps);
    for (int64_t i = 0; i < d; ++i) {
      float value = (input[i] - mean) * inv * weight[i];
      if (bias) value += bias[i];
      out[i] = value;
    }
  };
  if (cols > 1 && d * cols >= kParallelThreshold) {
    parallel_for(cols, [&](int64_t c0, int64_t c1) {
      for (int64_t c = c0; c < c1; ++c) normalize(y + c * d, x + c * d);
    });
  } else {
    for (int64_t c = 0; c < cols; ++c) normalize(y + c * d, x + c * d);
  }
}

// ---------------------------------------------------------------------------
// crates/cpu-kernels/src/lib.rs:516-538 -- geglu_into:
// out[i + I*c] = gelu_erf_f32(u[i + 2I*c]) * u[I + i + 2I*c].
// ---------------------------------------------------------------------------
void orc_geglu_f32(const float* u, int64_t inter, int64_t cols, float* out) {
  if (inter == 0 || cols == 0) return;
  auto activate = [&](const float* input, float* output) {
    for (int64_t i = 0; i < inter; ++i) output[i] = orc_gelu_erf_f32(input[i]) * input[inter + i];
  };
  if (cols > 1 && inter * cols >= (int64_t(1) << 14)) {
    parallel_for(cols, [&](int64_t c0, int64_t c1) {
      for (int64_t c = c0; c < c1; ++c) activate(u + 2 * inter * c, out + inter * c);
    });
  } else {
    for (int64_t c = 0; c < cols; ++c) activate(u + 2 * inter * c, out + inter * c);
  }
}

// ---------------------------------------------------------------------------
// crates/cpu-kernels/src/lib.rs:545-581 -- rms_norm_last_into. Column-major
// (rows, width): element (r, d) at r + rows*d. Note the multiply by the f32
// reciprocal of width (not a division).
// ---------------------------------------------------------------------------
void orc_rms_norm_last_f32(const float* x, int64_t rows, int64_t width, const float* weight,
                           int centered, float eps, float* out) {
  if (rows == 0 || width == 0) return;
  const float inv_width = 1.0f / float(width);
  parallel_for(rows, [&](int64_t r0, int64_t r1) {
    for (int64_t r = r0; r < r1; ++r) {
      float mean_sq = 0.0f;
      for (int64_t d = 0; d < width; ++d) {
        const float v = x[r + rows * d];
        mean_sq += v * v;
      }
      const float scale = 1.0f / std::sqrt(mean_sq * inv_width + eps);
      for (int64_t d = 0; d < width; ++d) {
        const float w = weight[d];
        const float wt = centered ? 1.0f + w : w;
        out[r + rows * d] = x[r + rows * d] * scale * wt;
      }
    }
  });
}

// ---------------------------------------------------------------------------
// crates/cpu-kernels/src/lib.rs:584-607 -- gated_silu_into, 4096-element tasks:
// out = (g / (1 + exp(-g))) * u.
// ---------------------------------------------------------------------------
void orc_gated_silu_f32(const float* gate, const float* up, float* out, int64_t n) {
  const int64_t per = 4096;
  parallel_for((n + per - 1) / per, [&](int64_t c0, int64_t c1) {
    for (int64_t c = c0; c < c1; ++c) {
      const int64_t end = std::min(n, (c + 1) * per);
      for (int64_t i = c * per; i < end; ++i) {
        const float g = gate[i];
        out[i] = (g / (1.0f + std::exp(-g))) * up[i];
      }
    }
  });
}

// ---------------------------------------------------------------------------
// Bias broadcast over feature-first (features, tokens) activations. In
// input_mul_weight_transpose_bias_into (cpu-kernels/src/lib.rs:274-288) the
// bias row is the SGEMM's initial accumulator (:284-286); as a standalone
// epilogue on a finished product the result is one rounding of x + bias[o].
// ---------------------------------------------------------------------------
void orc_bias_add_f32(const float* x, const float* bias, float* y, int64_t features,
                      int64_t tokens) {
  parallel_for(tokens, [&](int64_t t0, int64_t t1) {
    for (int64_t t = t0; t < t1; ++t)
      for (int64_t o = 0; o < features; ++o) y[o + features * t] = x[o + features * t] + bias[o];
  });
}

void orc_bias_act_f32(const float* x, const float* bias, float* y, int64_t features,
                      int64_t tokens, int act) {
  parallel_for(tokens, [&](int64_t t0, int64_t t1) {
    for (int64_t t = t0; t < t1; ++t)
      for (int64_t o = 0; o < features; ++o) {
        float v = x[o + features * t];
        if (bias) v = v + bias[o];
        if (act == 1) v = orc_gelu_erf_f32(v);
        else if (act == 2) v = v > 0.0f ? v : 0.0f;
        y[o + features * t] = v;
      }
  });
}

// crates/tenferro-ext/src/gemm_bias.rs:76-142 -> cpu-kernels lib.rs:274-288:
// x (in, length) and weight (in, out) column-major, y (out, length); the bias
// row is the initial accumulator, then y += x . W^T (summed here in index order;
// the reference's blocked SGEMM order is not observable, so this one is only
// tolerance-pinned).
void orc_gemm_bias_f32(const float* x, const float* weight, const float* bias, float* y,
                       int64_t in_dim, int64_t out_dim, int64_t length) {
  parallel_for(length, [&](int64_t t0, int64_t t1) {
    for (int64_t t = t0; t < t1; ++t)
      for (int64_t o = 0; o < out_dim; ++o) {
        float acc = bias[o];
        for (int64_t i = 0; i < in_dim; ++i) acc += x[i + in_dim * t] * weight[i + in_dim * o];
        y[o + out_dim * t] = acc;
      }
  });
}

void orc_add_f32(const float* a, const float* b, float* y, int64_t n) {
  parallel_for((n + 4095) / 4096, [&](int64_t c0, int64_t c1) {
    for (int64_t i = c0 * 4096; i < std::min(n, c1 * 4096); ++i) y[i] = a[i] + b[i];
  });
}

// ---------------------------------------------------------------------------
// Masked row softmax. EXCLUDE restates the f32 rows of
// crates/cpu-kernels/src/lib.rs:1053-1080 (GEMM path) and :1111-1153 (scalar
// path): kept scores are scaled, masked ones are -inf, the max uses `>`,
// non-finite values contribute 0, the sum is sequential, and each value is
// divided (not multiplied by a reciprocal) by the sum. FILL restates
// crates/tenferro-infer/src/softmax.rs:26-34 with util.rs:87 (-1e30 fill).
// Key masking: laya-infer/src/model.rs:474-483 (window, validity).
// ---------------------------------------------------------------------------
void orc_masked_softmax_f32(const float* scores, float* probs, int64_t batch, int64_t heads,
                            int64_t q_len, int64_t k_len, float scale, int semantics,
                            int causal, int64_t window, int window_skips_invalid_query,
                            int64_t valid_len, const int32_t* valid_lens,
                            const float* add_mask, int64_t add_sb, int64_t add_sq,
                            int64_t add_sk, const uint8_t* keep, int64_t keep_sb,
                            int64_t keep_sq, int64_t keep_sk) {
  const int64_t rows = batch * heads * q_len;
  parallel_for(rows, [&](int64_t r0, int64_t r1) {
    for (int64_t row = r0; row < r1; ++row) {
      const int64_t q = row % q_len;
      const int64_t b = row / (heads * q_len);
      const float* s = scores + row * k_len;
      float* p = probs + row * k_len;
      const int64_t vlen = valid_lens ? int64_t(valid_lens[b]) : valid_len;
      const bool q_valid = vlen < 0 || q < vlen;
      auto kept = [&](int64_t k) {
        if (vlen >= 0 && k >= vlen) return false;
        if (causal && k > q) return false;
        if (window >= 0 && !(window_skips_invalid_query && !q_valid)) {
          const int64_t diff = q > k ? q - k : k - q;
          if (diff > window) return false;
        }
        if (keep && keep[b * keep_sb + q * keep_sq + k * keep_sk] == 0) return false;
        return true;
      };
      if (semantics == 0) {
        float max = -std::numeric_limits<float>::infinity();
        for (int64_t k = 0; k < k_len; ++k) {
          float v;
          if (kept(k)) {
            v = s[k] * scale;
            if (add_mask) v = v + add_mask[b * add_sb + q * add_sq + k * add_sk];
          } else {
            v = -std::numeric_limits<float>::infinity();
          }
          p[k] = v;
          if (v > max) max = v;
        }
        float sum = 0.0f;
        for (int64_t k = 0; k < k_len; ++k) {
          const float e = std::isfinite(p[k]) ? std::exp(p[k] - max) : 0.0f;
          p[k] = e;
          sum += e;
        }
        for (int64_t k = 0; k < k_len; ++k) p[k] = p[k] / sum;
      } else {
        float max = -std::numeric_limits<float>::infinity();
        for (int64_t k = 0; k < k_len; ++k) {
          float v = s[k] * scale;
          if (add_mask) v = v + add_mask[b * add_sb + q * add_sq + k * add_sk];
          if (!kept(k)) v = -1.0e30f;
          p[k] = v;
          if (v > max) max = v;
        }
        float sum = 0.0f;
        for (int64_t k = 0; k < k_len; ++k) {
          const float e = std::exp(p[k] - max);
          p[k] = e;
          sum += e;
        }
        for (int64_t k = 0; k < k_len; ++k) p[k] = p[k] / sum;
      }
    }
  });
}

// ---------------------------------------------------------------------------
// RoPE, crates/tenferro-infer/src/rope.rs:68-113 (rotate_pair_half). The
// angle is (position as f64) * base.powf(-2 i / width) in f64 (:84-92); the
// f32 path rounds the f64 cos/sin to f32 (table(), :15-24). Pairs are
// (i, i + half): out1 = x1*cos - x2*sin, out2 = x1*sin + x2*cos, each product
// rounded (separate eager mul/sub/add ops).
// ---------------------------------------------------------------------------
void orc_rope_tables_f64(double base, int64_t seq, int64_t rotary_dim, double* cos_t,
                         double* sin_t) {
  const int64_t half = rotary_dim / 2;
  for (int64_t p = 0; p < seq; ++p)
    for (int64_t i = 0; i < half; ++i) {
      const double theta =
          double(p) * std::pow(base, -2.0 * double(i) / double(rotary_dim));
      cos_t[p * half + i] = std::cos(theta);
      sin_t[p * half + i] = std::sin(theta);
    }
}

void orc_rope_tables_f32(double base, int64_t seq, int64_t rotary_dim, float* cos_t,
                         float* sin_t) {
  const int64_t half = rotary_dim / 2;
  std::vector<double> c(size_t(seq * half)), s(size_t(seq * half));
  orc_rope_tables_f64(base, seq, rotary_dim, c.data(), s.data());
  for (int64_t k = 0; k < seq * half; ++k) {
    cos_t[k] = float(c[size_t(k)]);
    sin_t[k] = float(s[size_t(k)]);
  }
}

void orc_rope_pairhalf_f32(const float* x, float* y, const float* cos_t, const float* sin_t,
                           int64_t n_vec, int64_t seq, int64_t batch, int64_t head_dim,
                           int64_t rotary_dim, int64_t s_vec, int64_t s_pos, int64_t s_batch,
                           int64_t s_feat) {
  rope_impl<float>(x, y, cos_t, sin_t, n_vec, seq, batch, head_dim, rotary_dim, s_vec, s_pos,
                   s_batch, s_feat);
}

void orc_rope_pairhalf_f64(const double* x, double* y, const double* cos_t,
                           const double* sin_t, int64_t n_vec, int64_t seq, int64_t batch,
                           int64_t head_dim, int64_t rotary_dim, int64_t s_vec, int64_t s_pos,
                           int64_t s_batch, int64_t s_feat) {
  rope_impl<double>(x, y, cos_t, sin_t, n_vec, seq, batch, head_dim, rotary_dim, s_vec, s_pos,
                    s_batch, s_feat);
}

// ---------------------------------------------------------------------------
// Attention blocks, crates/cpu-kernels/src/lib.rs:618-760 (Jeff) and :819-1150
// (Laya). Products and sums are rounded one by one (no contraction), sums run
// in key / channel order, exp is glibc expf, as the Rust code compiles.
// ---------------------------------------------------------------------------
void orc_rope_tables_powf_f32(float base, int64_t seq, int64_t rotary_dim, float* cos_t,
                              float* sin_t) {
  const int64_t half = rotary_dim / 2;
  for (int64_t p = 0; p < seq; ++p)
    for (int64_t i = 0; i < half; ++i) {
      const float e = (-2.0f * float(i)) / float(rotary_dim);
      const float theta = float(p) * powf(base, e);
      cos_t[p * half + i] = cosf(theta);
      sin_t[p * half + i] = sinf(theta);
    }
}

}  // extern "C"

namespace {
// a*c - b*s and a*s + b*c for the pair (x[i], x[i + half]) of one row.
void rotate_row(float* x, const float* c, const float* s, int64_t half) {
  for (int64_t i = 0; i < half; ++i) {
    const float a = x[i], b = x[i + half];
    x[i] = a * c[i] - b * s[i];
    x[i + half] = a * s[i] + b * c[i];
  }
}

// Masked scaled dot-product attention of one head, scalar path of
// lib.rs:1106-1147 / :711-752. q, k, v (L, hd) row-major; keep(query, key);
// out_row(query) receives hd values (accumulated from 0, keys with p == 0
// skipped). divide: p = e / sum per key (Laya); else p computed the same way
// but an empty row leaves zeros (Jeff checks sum > 0 first).
template <class Keep, class OutRow>
void head_attention(const float* q, const float* k, const float* v, int64_t L, int64_t hd,
                    float scale, bool jeff, Keep keep, OutRow out_row) {
  std::vector<float> probs(static_cast<size_t>(L)), acc(static_cast<size_t>(hd));
  for (int64_t query = 0; query < L; ++query) {
    const float* qo = q + query * hd;
    float mx = -INFINITY;
    for (int64_t key = 0; key < L; ++key) {
      if (!keep(query, key)) {
        probs[size_t(key)] = -INFINITY;
        continue;
      }
      const float* ko = k + key * hd;
      float a = 0.0f;
      for (int64_t i = 0; i < hd; ++i) a += qo[i] * ko[i];
      const float score = a * scale;
      probs[size_t(key)] = score;
      if (score > mx) mx = score;
    }
    float sum = 0.0f;
    for (int64_t key = 0; key < L; ++key) {
      const float val = probs[size_t(key)];
      probs[size_t(key)] = std::isfinite(val) ? expf(val - mx) : 0.0f;
      sum += probs[size_t(key)];
    }
    for (int64_t i = 0; i < hd; ++i) acc[size_t(i)] = 0.0f;
    if (!jeff || sum > 0.0f) {
      for (int64_t key = 0; key < L; ++key) {
        const float p = probs[size_t(key)] / sum;
        if (p == 0.0f) continue;
        const float* vo = v + key * hd;
        for (int64_t i = 0; i < hd; ++i) acc[size_t(i)] += vo[i] * p;
      }
    }
    out_row(query, acc.data());
  }
}
}  // namespace

extern "C" {

void orc_laya_qkv_prep_f32(const float* qkv, const float* cos_t, const float* sin_t,
                           int64_t hidden, int64_t heads, int64_t length, int64_t batch,
                           float* qh, float* kh, float* vh) {
  const int64_t hd = hidden / heads, half = hd / 2;
  parallel_for(batch * heads, [&](int64_t h0, int64_t h1) {
    for (int64_t bh = h0; bh < h1; ++bh) {
      const int64_t b = bh / heads, head = bh % heads, feat = head * hd;
      for (int64_t l = 0; l < length; ++l) {
        const float* src = qkv + 3 * hidden * (l + length * b) + feat;
        const int64_t dst = (bh * length + l) * hd;
        for (int64_t i = 0; i < hd; ++i) {
          qh[dst + i] = src[i];
          kh[dst + i] = src[hidden + i];
          vh[dst + i] = src[2 * hidden + i];
        }
        if (cos_t) {
          rotate_row(qh + dst, cos_t + l * half, sin_t + l * half, half);
          rotate_row(kh + dst, cos_t + l * half, sin_t + l * half, half);
        }
      }
    }
  });
}

void orc_laya_attention_block_f32(const float* qkv, const uint8_t* keep, int64_t hidden,
                                  int64_t heads, int64_t length, int64_t batch,
                                  const float* cos_t, const float* sin_t, float* out) {
  const int64_t hd = hidden / heads, L = length;
  const float scale = 1.0f / sqrtf(float(hd));
  parallel_for(batch * heads, [&](int64_t h0, int64_t h1) {
    const size_t n = static_cast<size_t>(L * hd);
    std::vector<float> q(n), k(n), v(n);
    for (int64_t bh = h0; bh < h1; ++bh) {
      const int64_t b = bh / heads, head = bh % heads, feat = head * hd;
      for (int64_t l = 0; l < L; ++l) {
        const float* src = qkv + 3 * hidden * (l + L * b) + feat;
        for (int64_t i = 0; i < hd; ++i) {
          q[size_t(l * hd + i)] = src[i];
          k[size_t(l * hd + i)] = src[hidden + i];
          v[size_t(l * hd + i)] = src[2 * hidden + i];
        }
        if (cos_t) {
          rotate_row(q.data() + l * hd, cos_t + l * (hd / 2), sin_t + l * (hd / 2), hd / 2);
          rotate_row(k.data() + l * hd, cos_t + l * (hd / 2), sin_t + l * (hd / 2), hd / 2);
        }
      }
      head_attention(
          q.data(), k.data(), v.data(), L, hd, scale, false,
          [&](int64_t qi, int64_t ki) { return keep[qi + L * (ki + L * b)] != 0; },
          [&](int64_t qi, const float* acc) {
            float* o = out + feat + hidden * (qi + L * b);
            for (int64_t i = 0; i < hd; ++i) o[i] = acc[i];
          });
    }
  });
}

void orc_jeff_qkv_prep_f32(const float* q, const float* k, const float* v, const float* q_norm,
                           const float* k_norm, const float* cos_t, const float* sin_t,
                           int64_t length, int64_t heads, int64_t head_dim, int64_t rotary_dim,
                           float eps, float* qh, float* kh, float* vh) {
  const int64_t L = length, hd = head_dim, half = rotary_dim / 2;
  parallel_for(heads, [&](int64_t h0, int64_t h1) {
    for (int64_t head = h0; head < h1; ++head) {
      const int64_t feat = head * hd;
      for (int64_t t = 0; t < L; ++t) {
        const int64_t dst = (head * L + t) * hd;
        for (int64_t i = 0; i < hd; ++i) {
          qh[dst + i] = q[t + L * (feat + i)];
          kh[dst + i] = k[t + L * (feat + i)];
          vh[dst + i] = v[t + L * (feat + i)];
        }
        for (int which = 0; which < 2; ++which) {
          float* row = (which == 0 ? qh : kh) + dst;
          const float* w = which == 0 ? q_norm : k_norm;
          float mean_sq = 0.0f;
          for (int64_t i = 0; i < hd; ++i) mean_sq += row[i] * row[i];
          mean_sq /= float(hd);
          const float scale = 1.0f / sqrtf(mean_sq + eps);
          for (int64_t i = 0; i < hd; ++i) row[i] *= scale * (1.0f + w[i]);
          if (half > 0) rotate_row(row, cos_t + t * half, sin_t + t * half, half);
        }
      }
    }
  });
}

void orc_jeff_full_attention_f32(const float* q, const float* k, const float* v,
                                 const float* gate, const float* q_norm, const float* k_norm,
                                 const float* mask, int64_t length, int64_t heads,
                                 int64_t head_dim, int64_t rotary_dim, float theta, float eps,
                                 float* out) {
  const int64_t L = length, hd = head_dim, half = rotary_dim / 2;
  std::vector<float> c(size_t(std::max<int64_t>(1, L * half))), s(c.size());
  if (half > 0) orc_rope_tables_powf_f32(theta, L, rotary_dim, c.data(), s.data());
  std::vector<float> qh(static_cast<size_t>(heads * L * hd)), kh(qh.size()), vh(qh.size());
  orc_jeff_qkv_prep_f32(q, k, v, q_norm, k_norm, c.data(), s.data(), L, heads, hd, rotary_dim,
                        eps, qh.data(), kh.data(), vh.data());
  const float scale = 1.0f / sqrtf(float(hd));
  parallel_for(heads, [&](int64_t h0, int64_t h1) {
    for (int64_t head = h0; head < h1; ++head) {
      const int64_t feat = head * hd, base = head * L * hd;
      head_attention(
          qh.data() + base, kh.data() + base, vh.data() + base, L, hd, scale, true,
          [&](int64_t qi, int64_t ki) { return ki <= qi && mask[ki] != 0.0f; },
          [&](int64_t qi, const float* acc) {
            for (int64_t i = 0; i < hd; ++i) {
              const float g = gate[qi + L * (feat + i)];
              const float sig = 1.0f / (1.0f + expf(-g));
              out[qi + L * (feat + i)] = acc[i] * sig;
            }
          });
    }
  });
}

// ---------------------------------------------------------------------------
// Token embedding gather, crates/tenferro-ext/src/cuda/fused.cu:304-318 with
// the strides FusedScope passes (cuda_fused.rs:821-863).
// ---------------------------------------------------------------------------
void orc_embedding_f32(const float* table, const int64_t* ids, float* out, int64_t hidden,
                       int64_t length, int64_t o_tok, int64_t o_feat, int64_t t_feat,
                       int64_t t_tok) {
  for (int64_t f = 0; f < hidden; ++f)
    for (int64_t t = 0; t < length; ++t)
      out[t * o_tok + f * o_feat] = table[f * t_feat + ids[t] * t_tok];
}

// ---------------------------------------------------------------------------
// crates/tenferro-ext/src/lib.rs:273-285 -- erf_f64, Abramowitz-Stegun 7.1.26.
// ---------------------------------------------------------------------------
double orc_erf_f64(double x) {
  if (x == 0.0) return 0.0;
  const double sign = x < 0.0 ? -1.0 : 1.0;
  x = std::fabs(x);
  const double t = 1.0 / (1.0 + 0.3275911 * x);
  const double poly =
      ((((1.061405429 * t - 1.453152027) * t + 1.421413741) * t - 0.284496736) * t +
       0.254829592) *
      t;
  return sign * (1.0 - poly * std::exp(-x * x));
}

void orc_erf_f64_n(const double* x, double* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = orc_erf_f64(x[i]);
}

// crates/tenferro-ext/src/lib.rs:224-234 -- gelu_erf on a CPU session:
// scaled = x * FRAC_1_SQRT_2; gate = erf(scaled) + 1; half = x * 0.5; half * gate.
void orc_gelu_erf_f64_n(const double* x, double* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    const double scaled = x[i] * 0.70710678118654752440;
    const double gate = orc_erf_f64(scaled) + 1.0;
    const double half = x[i] * 0.5;
    y[i] = half * gate;
  }
}

// ---------------------------------------------------------------------------
// crates/tenferro-infer/src/norm.rs:11-45 -- layer_norm (f64), applied to the
// feature axis of a feature-first (d, cols) activation (the transpose pair of
// laya-infer/src/model.rs:1083-1096 only moves data). mean = sum * (1/width),
// var = sum((x-mean)^2) * (1/width), inv = 1/sqrt(var + eps).
// ---------------------------------------------------------------------------
void orc_layer_norm_feature_first_f64(const double* x, int64_t d, int64_t cols,
                                      const double* weight, const double* bias, double eps,
                                      double* y) {
  const double inv_width = 1.0 / double(d);
  parallel_for(cols, [&](int64_t c0, int64_t c1) {
    for (int64_t c = c0; c < c1; ++c) {
      const double* in = x + c * d;
      double* out = y + c * d;
      double sum = 0.0;
      for (int64_t i = 0; i < d; ++i) sum += in[i];
      const double mean = sum * inv_width;
      double sq = 0.0;
      for (int64_t i = 0; i < d; ++i) {
        const double centered = in[i] - mean;
        sq += centered * centered;
      }
      const double var = sq * inv_width;
      const double inv = 1.0 / std::sqrt(var + eps);
      for (int64_t i = 0; i < d; ++i) {
        double v = ((in[i] - mean) * inv) * weight[i];
        if (bias) v = v + bias[i];
        out[i] = v;
      }
    }
  });
}

// crates/tenferro-infer/src/norm.rs:52-103 -- rms_norm (f64) over the last
// axis of a column-major (rows, width) activation.
void orc_rms_norm_last_f64(const double* x, int64_t rows, int64_t width, const double* weight,
                           int centered, double eps, double* out) {
  const double inv_width = 1.0 / double(width);
  parallel_for(rows, [&](int64_t r0, int64_t r1) {
    for (int64_t r = r0; r < r1; ++r) {
      double sq = 0.0;
      for (int64_t d = 0; d < width; ++d) sq += x[r + rows * d] * x[r + rows * d];
      const double inv = 1.0 / std::sqrt(sq * inv_width + eps);
      for (int64_t d = 0; d < width; ++d) {
        const double scale = centered ? weight[d] + 1.0 : weight[d];
        out[r + rows * d] = (x[r + rows * d] * inv) * scale;
      }
    }
  });
}

// crates/tenferro-infer/src/softmax.rs:8-21 -- softmax (f64) over contiguous rows.
void orc_softmax_rows_f64(const double* x, double* y, int64_t rows, int64_t cols) {
  parallel_for(rows, [&](int64_t r0, int64_t r1) {
    for (int64_t r = r0; r < r1; ++r) {
      const double* in = x + r * cols;
      double* out = y + r * cols;
      double max = -std::numeric_limits<double>::infinity();
      for (int64_t k = 0; k < cols; ++k) max = std::max(max, in[k]);
      double sum = 0.0;
      for (int64_t k = 0; k < cols; ++k) {
        out[k] = std::exp(in[k] - max);
        sum += out[k];
      }
      for (int64_t k = 0; k < cols; ++k) out[k] = out[k] / sum;
    }
  });
}

}  // extern "C"
