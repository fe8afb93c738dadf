// ORACLE / TEST INFRASTRUCTURE — never linked into the product library.
//
// CPU restatement of the Metal kernels the GPT decoder dispatches.  Used by
// both oracle builds: the stand-alone port (gpt_port.cpp) and the CPU
// MetalContext shim that the reference's own gpt.cpp / gpt_sampling.cpp are
// compiled against (ref_shim.cpp).
//
// Precision choice: every reduction (LayerNorm statistics, dot products,
// softmax) is carried in double and rounded to float once per output, so the
// oracle is closer to the exact value than any fp32 device ordering.  Values
// stored between ops are float, as in the reference.  Each function names the
// Metal kernel (vendor/metal-runtime/metal/kernels.metal) whose math it restates.
#pragma once

#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstdlib>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace orc {

// ---------------------------------------------------------------- thread pool
// Work is split into contiguous index ranges; every output element is produced
// by exactly one thread with a fixed sequential order, so results do not depend
// on the thread count.
class Pool {
public:
    explicit Pool(int n) : n_(std::max(1, n)) {
        for (int i = 1; i < n_; ++i) workers_.emplace_back([this, i] { loop(i); });
    }
    ~Pool() {
        {
            std::lock_guard<std::mutex> g(m_);
            stop_ = true;
            ++gen_;
        }
        cv_.notify_all();
        for (auto& t : workers_) t.join();
    }
    int size() const { return n_; }
    void run(size_t n, const std::function<void(size_t, size_t)>& fn, size_t min_chunk = 1) {
        const size_t parts = std::min<size_t>(n_, std::max<size_t>(1, n / std::max<size_t>(1, min_chunk)));
        if (parts <= 1) {
            if (n) fn(0, n);
            return;
        }
        std::unique_lock<std::mutex> lk(m_);
        fn_ = &fn;
        total_ = n;
        parts_ = parts;
        pending_ = static_cast<int>(parts) - 1;
        ++gen_;
        lk.unlock();
        cv_.notify_all();
        fn(0, n / parts);
        lk.lock();
        done_cv_.wait(lk, [this] { return pending_ == 0; });
        fn_ = nullptr;
    }

private:
    void loop(int idx) {
        uint64_t seen = 0;
        for (;;) {
            std::unique_lock<std::mutex> lk(m_);
            cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
            if (stop_) return;
            seen = gen_;
            if (static_cast<size_t>(idx) >= parts_ || !fn_) continue;
            const auto* fn = fn_;
            const size_t b = total_ * idx / parts_, e = total_ * (idx + 1) / parts_;
            lk.unlock();
            (*fn)(b, e);
            lk.lock();
            if (--pending_ == 0) done_cv_.notify_all();
        }
    }
    int n_;
    std::vector<std::thread> workers_;
    std::mutex m_;
    std::condition_variable cv_, done_cv_;
    const std::function<void(size_t, size_t)>* fn_ = nullptr;
    size_t total_ = 0, parts_ = 0;
    int pending_ = 0;
    uint64_t gen_ = 0;
    bool stop_ = false;
};

inline int default_threads() {
    if (const char* v = std::getenv("ORC_THREADS")) {
        const int n = std::atoi(v);
        if (n > 0) return n;
    }
    const unsigned hc = std::thread::hardware_concurrency();
    return hc ? static_cast<int>(hc) : 1;
}

inline Pool& pool() {
    static Pool p(default_threads());
    return p;
}

// --------------------------------------------------------------- dot products
inline double dot_d(const float* a, const float* b, uint32_t n) {
    double acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    uint32_t i = 0;
    for (; i + 8 <= n; i += 8)
        for (int j = 0; j < 8; ++j) acc[j] += double(a[i + j]) * double(b[i + j]);
    for (; i < n; ++i) acc[0] += double(a[i]) * double(b[i]);
    return ((acc[0] + acc[4]) + (acc[1] + acc[5])) + ((acc[2] + acc[6]) + (acc[3] + acc[7]));
}

// Four dot products sharing the row `w` (keeps the weight row in L1 across tokens).
inline void dot_d4(const float* w, const float* x0, const float* x1, const float* x2, const float* x3,
                   uint32_t n, double out[4]) {
    double a0[4] = {0, 0, 0, 0}, a1[4] = {0, 0, 0, 0}, a2[4] = {0, 0, 0, 0}, a3[4] = {0, 0, 0, 0};
    uint32_t i = 0;
    for (; i + 4 <= n; i += 4)
        for (int j = 0; j < 4; ++j) {
            const double wv = w[i + j];
            a0[j] += wv * x0[i + j];
            a1[j] += wv * x1[i + j];
            a2[j] += wv * x2[i + j];
            a3[j] += wv * x3[i + j];
        }
    for (; i < n; ++i) {
        const double wv = w[i];
        a0[0] += wv * x0[i];
        a1[0] += wv * x1[i];
        a2[0] += wv * x2[i];
        a3[0] += wv * x3[i];
    }
    out[0] = (a0[0] + a0[2]) + (a0[1] + a0[3]);
    out[1] = (a1[0] + a1[2]) + (a1[1] + a1[3]);
    out[2] = (a2[0] + a2[2]) + (a2[1] + a2[3]);
    out[3] = (a3[0] + a3[2]) + (a3[1] + a3[3]);
}

// ------------------------------------------------------------------- kernels
// y[t, r] = W[r, :] . x[t, :] + b[r]   (W row-major [rows, cols]).
// Restates mit2_linear_gemv_f32 (kernels.metal:1054-1081) for one token and the
// MPS GEMM path with the bias broadcast into C (metal_context.mm:368-410).
inline void linear_rows(const float* W, const float* b, const float* x, uint32_t tokens,
                        uint32_t rows, uint32_t cols, float* y) {
    pool().run(rows, [&](size_t r0, size_t r1) {
        for (size_t r = r0; r < r1; ++r) {
            const float* w = W + r * cols;
            uint32_t t = 0;
            for (; t + 4 <= tokens; t += 4) {
                double d[4];
                dot_d4(w, x + size_t(t) * cols, x + size_t(t + 1) * cols, x + size_t(t + 2) * cols,
                       x + size_t(t + 3) * cols, cols, d);
                for (int j = 0; j < 4; ++j) y[size_t(t + j) * rows + r] = float(d[j] + double(b[r]));
            }
            for (; t < tokens; ++t)
                y[size_t(t) * rows + r] = float(dot_d(w, x + size_t(t) * cols, cols) + double(b[r]));
        }
    }, 16);
}

// Restates mit2_layernorm_f32_rows (kernels.metal:618-669): two-pass mean then
// centred biased variance, eps inside the square root.
inline void layernorm_rows(const float* x, const float* g, const float* be, uint32_t tokens,
                           uint32_t width, float eps, float* out) {
    for (uint32_t t = 0; t < tokens; ++t) {
        const float* r = x + size_t(t) * width;
        double s = 0;
        for (uint32_t i = 0; i < width; ++i) s += r[i];
        const double mean = s / width;
        double v = 0;
        for (uint32_t i = 0; i < width; ++i) {
            const double d = double(r[i]) - mean;
            v += d * d;
        }
        const double inv = 1.0 / std::sqrt(v / width + double(eps));
        float* o = out + size_t(t) * width;
        for (uint32_t i = 0; i < width; ++i) o[i] = float((double(r[i]) - mean) * inv * g[i] + be[i]);
    }
}

// Restates mit2_gelu_f32 (kernels.metal:486-503): tanh GELU with the identity
// above 10 and zero below -10.
inline float gelu(float v) {
    if (v > 10.0f) return v;
    if (v < -10.0f) return 0.0f;
    const double d = v;
    return float(0.5 * d * (1.0 + std::tanh(0.7978845608028654 * (d + 0.044715 * d * d * d))));
}

// Restates mit2_gpt_causal_attention_sgq_f32 (kernels.metal:2249-2290): packed
// qkv [tokens, 3*width] (q | k | v, head h at h*head_dim), causal softmax with
// scale rsqrt(head_dim), output [tokens, width].
inline void causal_attention(const float* qkv, uint32_t tokens, uint32_t heads, uint32_t head_dim,
                             float* out) {
    const uint32_t width = heads * head_dim, qw = 3 * width;
    const double scale = 1.0 / std::sqrt(double(head_dim));
    pool().run(size_t(heads) * tokens, [&](size_t b, size_t e) {
        std::vector<double> p(tokens), acc(head_dim);
        for (size_t job = b; job < e; ++job) {
            const uint32_t h = uint32_t(job / tokens), tq = uint32_t(job % tokens);
            const float* q = qkv + size_t(tq) * qw + h * head_dim;
            double m = -INFINITY;
            for (uint32_t tk = 0; tk <= tq; ++tk) {
                const float* k = qkv + size_t(tk) * qw + width + h * head_dim;
                p[tk] = dot_d(q, k, head_dim) * scale;
                m = std::max(m, p[tk]);
            }
            double l = 0;
            std::fill(acc.begin(), acc.end(), 0.0);
            for (uint32_t tk = 0; tk <= tq; ++tk) {
                const double w = std::exp(p[tk] - m);
                l += w;
                const float* v = qkv + size_t(tk) * qw + 2 * width + h * head_dim;
                for (uint32_t d = 0; d < head_dim; ++d) acc[d] += w * v[d];
            }
            float* o = out + size_t(tq) * width + h * head_dim;
            for (uint32_t d = 0; d < head_dim; ++d) o[d] = float(acc[d] / l);
        }
    });
}

// Restates mit2_gpt_cached_attention_resident_f32 (kernels.metal:2064-2145):
// one query (q of `qkv`) against cache_tokens cached keys plus the current key
// (taken from `qkv`), cache layout [tokens, width].  The append of the current
// K/V into the cache is done by the caller.
inline void cached_attention(const float* cache_k, const float* cache_v, const float* qkv,
                             uint32_t cache_tokens, uint32_t heads, uint32_t head_dim, float* out) {
    const uint32_t width = heads * head_dim, keys = cache_tokens + 1;
    const double scale = 1.0 / std::sqrt(double(head_dim));
    pool().run(heads, [&](size_t b, size_t e) {
        std::vector<double> p(keys), acc(head_dim);
        for (size_t h = b; h < e; ++h) {
            const float* q = qkv + h * head_dim;
            double m = -INFINITY;
            for (uint32_t tk = 0; tk < keys; ++tk) {
                const float* k = tk < cache_tokens ? cache_k + size_t(tk) * width + h * head_dim
                                                   : qkv + width + h * head_dim;
                p[tk] = dot_d(q, k, head_dim) * scale;
                m = std::max(m, p[tk]);
            }
            double l = 0;
            std::fill(acc.begin(), acc.end(), 0.0);
            for (uint32_t tk = 0; tk < keys; ++tk) {
                const double w = std::exp(p[tk] - m);
                l += w;
                const float* v = tk < cache_tokens ? cache_v + size_t(tk) * width + h * head_dim
                                                   : qkv + 2 * width + h * head_dim;
                for (uint32_t d = 0; d < head_dim; ++d) acc[d] += w * v[d];
            }
            for (uint32_t d = 0; d < head_dim; ++d) out[h * head_dim + d] = float(acc[d] / l);
        }
    });
}

// Conv1D [in, out] -> row-major [out, in] (the transpose gpt.cpp:24-33 caches).
inline std::vector<float> transpose(const float* raw, size_t in, size_t out_cols) {
    std::vector<float> t(in * out_cols);
    pool().run(out_cols, [&](size_t c0, size_t c1) {
        for (size_t c = c0; c < c1; ++c)
            for (size_t i = 0; i < in; ++i) t[c * in + i] = raw[i * out_cols + c];
    }, 64);
    return t;
}

}  // namespace orc
