// CPU oracle: C++ restatement of rtensor's CPU backend.  TEST INFRASTRUCTURE
// ONLY -- see rtensor_cpu.h.  Compiled with -ffp-contract=off so that every
// `a * b + c` rounds twice, as the Rust reference does.
#include "rtensor_cpu.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

namespace {

// ---------------------------------------------------------------- Rng
// xorshift64* (crates/rtensor/src/rng.rs:12-20).
inline uint64_t next_u64(uint64_t* s) {
    uint64_t x = *s;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *s = x;
    return x * 0x2545F4914F6CDD1DULL;
}
// rng.rs:22-24: (next >> 40) as f32 / 2^24.
inline float uniform(uint64_t* s) { return (float)(next_u64(s) >> 40) / (float)(1ULL << 24); }
// rng.rs:27-29: lo + u * (hi - lo).
inline float range(uint64_t* s, float lo, float hi) { return lo + uniform(s) * (hi - lo); }
// rng.rs:32-36: Box-Muller in f32 (ln/cos/sqrt resolve to the same libm calls
// as Rust's f32::ln / f32::cos / f32::sqrt on Linux).
inline float normal(uint64_t* s) {
    float u1 = std::max(uniform(s), 1e-7f);
    float u2 = uniform(s);
    const float PI = 3.14159265358979323846f;
    return std::sqrt(-2.0f * std::log(u1)) * std::cos(2.0f * PI * u2);
}

// f32::powi with a runtime exponent lowers to compiler-rt's __powisf2:
// square-and-multiply over the exponent bits.
inline float powi_f32(float a, int b) {
    bool recip = b < 0;
    float r = 1.0f;
    for (;;) {
        if (b & 1) r *= a;
        b /= 2;
        if (b == 0) break;
        a *= a;
    }
    return recip ? 1.0f / r : r;
}

// Round an f32 to the nearest bf16 (ties to even) and widen it back.
inline float round_bf16(float f) {
    uint32_t b;
    std::memcpy(&b, &f, 4);
    b = (b + (((b >> 16) & 1u) + 0x7FFFu)) & 0xFFFF0000u;
    float r;
    std::memcpy(&r, &b, 4);
    return r;
}
inline void round_bf16(std::vector<float>& v) {
    for (auto& x : v) x = round_bf16(x);
}

// ---------------------------------------------------------------- matmul
// Rows [r0, r1) of C = A B, ikj order (tensor.rs:318-373).
void matmul_rows(const float* a, const float* b, float* c, size_t r0, size_t r1, size_t k, size_t n) {
    if (k * n <= 32768) {
        for (size_t i = r0; i < r1; ++i) {
            float* dst = c + i * n;
            const float* arow = a + i * k;
            for (size_t p = 0; p < k; ++p) {
                float av = arow[p];
                if (av == 0.0f) continue;
                const float* brow = b + p * n;
                for (size_t j = 0; j < n; ++j) dst[j] += av * brow[j];
            }
        }
        return;
    }
    const size_t JC = 256, PC = 128;
    for (size_t j0 = 0; j0 < n; j0 += JC) {
        size_t j1 = std::min(j0 + JC, n);
        for (size_t p0 = 0; p0 < k; p0 += PC) {
            size_t p1 = std::min(p0 + PC, k);
            for (size_t i = r0; i < r1; ++i) {
                const float* arow = a + i * k;
                float* dst = c + i * n;
                for (size_t p = p0; p < p1; ++p) {
                    float av = arow[p];
                    if (av == 0.0f) continue;
                    const float* brow = b + p * n;
                    for (size_t j = j0; j < j1; ++j) dst[j] += av * brow[j];
                }
            }
        }
    }
}

void matmul(const float* a, const float* b, float* c, size_t m, size_t k, size_t n, int threads) {
    std::memset(c, 0, sizeof(float) * m * n);
    if (m == 0 || n == 0 || k == 0) return;
    if (threads > 1 && m >= (size_t)threads) {
        // Split the row loop: every output element keeps its p-ascending
        // summation order, so the result does not depend on `threads`.
        std::vector<std::thread> pool;
        size_t nt = (size_t)threads;
        for (size_t t = 0; t < nt; ++t) {
            size_t r0 = m * t / nt, r1 = m * (t + 1) / nt;
            pool.emplace_back(matmul_rows, a, b, c, r0, r1, k, n);
        }
        for (auto& th : pool) th.join();
        return;
    }
    matmul_rows(a, b, c, 0, m, k, n);
}

// tensor.rs:132-155, 32x32 blocks.
void transpose(const float* a, float* out, size_t r, size_t c) {
    const size_t T = 32;
    for (size_t i0 = 0; i0 < r; i0 += T) {
        size_t i1 = std::min(i0 + T, r);
        for (size_t j0 = 0; j0 < c; j0 += T) {
            size_t j1 = std::min(j0 + T, c);
            for (size_t i = i0; i < i1; ++i)
                for (size_t j = j0; j < j1; ++j) out[j * r + i] = a[i * c + j];
        }
    }
}

// tensor.rs:410-418: out += G[i,:] for i = 0..n-1.
void reduce_rows(const float* g, float* out, size_t n, size_t m) {
    std::memset(out, 0, sizeof(float) * m);
    for (size_t i = 0; i < n; ++i)
        for (size_t j = 0; j < m; ++j) out[j] += g[i * m + j];
}

// tensor.rs:455-472.
void softmax_rows(const float* z, float* out, size_t r, size_t c) {
    for (size_t i = 0; i < r; ++i) {
        const float* row = z + i * c;
        float* dst = out + i * c;
        float mx = -INFINITY;
        for (size_t j = 0; j < c; ++j) mx = std::fmax(mx, row[j]);
        float sum = 0.0f;
        for (size_t j = 0; j < c; ++j) {
            float e = std::exp(row[j] - mx);
            dst[j] = e;
            sum += e;
        }
        for (size_t j = 0; j < c; ++j) dst[j] /= sum;
    }
}

// losses.rs:99-115.  Value: -(1/n) sum y ln max(p, 1e-12); adjoint
// (P - Y) scaled by g/n with g = 1 (`probs.sub(&y).scale(g.item() / batch)`).
float softmax_xent(const float* logits, const float* onehot, size_t n, size_t c, float* dlogits) {
    std::vector<float> probs(n * c);
    softmax_rows(logits, probs.data(), n, c);
    float batch = (float)n;
    float total = 0.0f;
    for (size_t i = 0; i < n * c; ++i) {
        float y = onehot[i];
        if (y != 0.0f) total -= y * std::log(std::fmax(probs[i], 1e-12f));
    }
    if (dlogits) {
        float k = 1.0f / batch;
        for (size_t i = 0; i < n * c; ++i) dlogits[i] = (probs[i] - onehot[i]) * k;
    }
    return total / batch;
}

}  // namespace

// =================================================================== C API
extern "C" {

uint64_t or_rng_seed(uint64_t seed) { return seed == 0 ? 0x9E3779B97F4A7C15ULL : seed; }
void or_rng_uniform(uint64_t* s, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = uniform(s);
}
void or_rng_range(uint64_t* s, float lo, float hi, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = range(s, lo, hi);
}
void or_rng_normal(uint64_t* s, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = normal(s);
}
void or_rng_below(uint64_t* s, uint64_t n, uint32_t* out, size_t count) {
    for (size_t i = 0; i < count; ++i) out[i] = (uint32_t)(next_u64(s) % n);
}

void or_matmul(const float* a, const float* b, float* c, size_t m, size_t k, size_t n, int threads) {
    matmul(a, b, c, m, k, n, threads);
}
void or_transpose(const float* a, float* out, size_t r, size_t c) { transpose(a, out, r, c); }
void or_reduce_rows(const float* g, float* out, size_t n, size_t m) { reduce_rows(g, out, n, m); }
void or_softmax_rows(const float* z, float* out, size_t r, size_t c) { softmax_rows(z, out, r, c); }
float or_softmax_xent(const float* logits, const float* onehot, size_t n, size_t c, float* dlogits) {
    return softmax_xent(logits, onehot, n, c, dlogits);
}
void or_one_hot(const uint32_t* labels, size_t n, size_t classes, float* out) {
    std::memset(out, 0, sizeof(float) * n * classes);
    for (size_t i = 0; i < n; ++i) out[i * classes + labels[i]] = 1.0f;
}

// optim.rs:163-198: one fused loop with pre-inverted bias corrections.
void or_adam_update(float* theta, float* m, float* v, const float* g, size_t n,
                    float lr, float beta1, float beta2, float eps, int t) {
    float c1 = 1.0f - powi_f32(beta1, t);
    float c2 = 1.0f - powi_f32(beta2, t);
    float inv_c1 = 1.0f / c1, inv_c2 = 1.0f / c2;
    float omb1 = 1.0f - beta1, omb2 = 1.0f - beta2;
    for (size_t i = 0; i < n; ++i) {
        float gi = g[i];
        m[i] = m[i] * beta1 + gi * omb1;
        v[i] = v[i] * beta2 + (gi * gi) * omb2;
        float m_hat = m[i] * inv_c1;
        float v_hat = v[i] * inv_c2;
        theta[i] -= (m_hat / (std::sqrt(v_hat) + eps)) * lr;
    }
}

// optim.rs:80-115.
void or_sgd_update(float* theta, float* vel, const float* g, size_t n, float lr, float momentum) {
    if (momentum == 0.0f) {
        for (size_t i = 0; i < n; ++i) theta[i] -= g[i] * lr;
        return;
    }
    for (size_t i = 0; i < n; ++i) vel[i] = vel[i] * momentum + g[i] * lr;
    for (size_t i = 0; i < n; ++i) theta[i] -= vel[i];
}

}  // extern "C"

// ------------------------------------------------------------------ MLP
struct or_mlp {
    int L = 0;
    std::vector<size_t> dims;
    std::vector<std::vector<float>> W, b, dW, db;
    std::vector<std::vector<float>> mW, vW, mb, vb, velW, velb;
    std::vector<std::vector<float>> act;  // act[0] = x, act[l+1] = output of layer l
    size_t n = 0;
    int t = 0;
    int round = 0;                       // OR_ROUND_* / OR_SPLIT_ACT flags (bf16 emulation)
    std::vector<std::vector<float>> Wq;  // bf16-rounded weights (OR_ROUND_W)
    std::vector<std::vector<float>> fwd_in;  // OR_SPLIT_ACT: hi + lo of act[l], the next forward's input
};

extern "C" {

or_mlp* or_mlp_new(int n_layers, const size_t* dims) {
    or_mlp* m = new or_mlp;
    m->L = n_layers;
    m->dims.assign(dims, dims + n_layers + 1);
    for (int l = 0; l < n_layers; ++l) {
        size_t d = dims[l], u = dims[l + 1];
        m->W.emplace_back(d * u, 0.0f);
        m->b.emplace_back(u, 0.0f);
        m->dW.emplace_back(d * u, 0.0f);
        m->db.emplace_back(u, 0.0f);
    }
    return m;
}

void or_mlp_free(or_mlp* m) { delete m; }

void or_mlp_set(or_mlp* m, int l, const float* w, const float* b) {
    if (w) std::memcpy(m->W[l].data(), w, sizeof(float) * m->W[l].size());
    if (b) std::memcpy(m->b[l].data(), b, sizeof(float) * m->b[l].size());
}
void or_mlp_get(const or_mlp* m, int l, float* w, float* b) {
    if (w) std::memcpy(w, m->W[l].data(), sizeof(float) * m->W[l].size());
    if (b) std::memcpy(b, m->b[l].data(), sizeof(float) * m->b[l].size());
}
void or_mlp_get_grads(const or_mlp* m, int l, float* dw, float* db) {
    if (dw) std::memcpy(dw, m->dW[l].data(), sizeof(float) * m->dW[l].size());
    if (db) std::memcpy(db, m->db[l].data(), sizeof(float) * m->db[l].size());
}
void or_mlp_get_logits(const or_mlp* m, float* out) {
    const auto& z = m->act[m->L];
    std::memcpy(out, z.data(), sizeof(float) * z.size());
}

// nn.rs:122-130: limit = sqrt(6 / (in + units)); W drawn row-major with
// Rng::range(-limit, limit); b = 0.
void or_mlp_init_glorot(or_mlp* m, uint64_t* s) {
    for (int l = 0; l < m->L; ++l) {
        size_t d = m->dims[l], u = m->dims[l + 1];
        float limit = std::sqrt(6.0f / (float)(d + u));
        for (auto& w : m->W[l]) w = range(s, -limit, limit);
        std::fill(m->b[l].begin(), m->b[l].end(), 0.0f);
    }
}

void or_mlp_init_kaiming(or_mlp* m, uint64_t* s) {
    for (int l = 0; l < m->L; ++l) {
        size_t d = m->dims[l];
        float limit = std::sqrt(6.0f / (float)d);
        for (auto& w : m->W[l]) w = range(s, -limit, limit);
        std::fill(m->b[l].begin(), m->b[l].end(), 0.0f);
    }
}

// Sequential::forward (nn.rs:179-181) of Dense layers (nn.rs:143-149):
// Z = x.matmul(W).add(b) (zip with b tiled over rows, tensor.rs:196-200),
// then relu (ops.rs:190-194) on hidden layers; the last layer is Linear.
static const float* gemm_weights(or_mlp* m, int l) {
    return (m->round & OR_ROUND_W) ? m->Wq[l].data() : m->W[l].data();
}

// Input of layer l's forward GEMM: x, the previous activation, or (split
// activations, hidden layer l) its hi + lo pair summed in f32, which is exact.
static const float* forward_input(or_mlp* m, int l) {
    return (l > 0 && l + 1 < m->L && (m->round & OR_SPLIT_ACT)) ? m->fwd_in[l].data() : m->act[l].data();
}

static void forward_impl(or_mlp* m, const float* x, size_t n, int threads) {
    m->n = n;
    m->act.resize(m->L + 1);
    m->act[0].assign(x, x + n * m->dims[0]);
    if (m->round & OR_ROUND_X) round_bf16(m->act[0]);
    if (m->round & OR_ROUND_W) {
        m->Wq.resize(m->L);
        for (int l = 0; l < m->L; ++l) {
            m->Wq[l] = m->W[l];
            round_bf16(m->Wq[l]);
        }
    }
    if (m->round & OR_SPLIT_ACT) m->fwd_in.resize(m->L);
    for (int l = 0; l < m->L; ++l) {
        size_t d = m->dims[l], u = m->dims[l + 1];
        auto& out = m->act[l + 1];
        out.resize(n * u);
        matmul(forward_input(m, l), gemm_weights(m, l), out.data(), n, d, u, threads);
        const float* bb = m->b[l].data();
        for (size_t i = 0; i < n; ++i)
            for (size_t j = 0; j < u; ++j) out[i * u + j] = out[i * u + j] + bb[j];
        if (l + 1 < m->L) {
            for (auto& v : out) v = std::fmax(v, 0.0f);
            if (m->round & OR_SPLIT_ACT) {
                auto& in = m->fwd_in[l + 1];
                in.resize(n * u);
                for (size_t i = 0; i < n * u; ++i) {
                    const float hi = round_bf16(out[i]);
                    in[i] = hi + round_bf16(out[i] - hi);
                    out[i] = hi;
                }
            } else if (m->round & OR_ROUND_ACT) {
                round_bf16(out);
            }
        }
    }
}

void or_mlp_set_rounding(or_mlp* m, int flags) { m->round = flags; }

void or_mlp_set_bf16_emulation(or_mlp* m, int on) {
    m->round = on ? (OR_ROUND_X | OR_ROUND_W | OR_ROUND_ACT | OR_ROUND_DELTA) : 0;
}

float or_mlp_forward(or_mlp* m, const float* x, const uint32_t* labels, size_t n, int threads) {
    forward_impl(m, x, n, threads);
    if (!labels) return 0.0f;
    size_t c = m->dims[m->L];
    std::vector<float> y(n * c);
    or_one_hot(labels, n, c, y.data());
    return softmax_xent(m->act[m->L].data(), y.data(), n, c, nullptr);
}

// One reference training step.  The backward pass is the tape's reverse sweep
// (tape.rs:197-226) over the nodes Dense::forward records: for each layer,
// from the last one down,
//   relu node:   g <- g * 1[A > 0]                    (ops.rs:190-194)
//   add node:    db = g.reduce_to([1,m])               (ops.rs:49-53)
//   matmul node: (g.matmul(&W.t()), x.t().matmul(g))  (ops.rs:125-129)
// Every parent receives exactly one adjoint in a Sequential MLP, so no
// accumulation happens.  Then Optimizer::step over [W1, b1, W2, b2, ...].
float or_mlp_train_step(or_mlp* m, const float* x, const uint32_t* labels, size_t n,
                        int optimizer, float lr, int threads, int input_grad) {
    forward_impl(m, x, n, threads);
    const int L = m->L;
    size_t c = m->dims[L];
    std::vector<float> y(n * c);
    or_one_hot(labels, n, c, y.data());
    std::vector<float> g(n * c);
    float loss = softmax_xent(m->act[L].data(), y.data(), n, c, g.data());
    const bool round_delta = (m->round & OR_ROUND_DELTA) != 0;
    if (round_delta) round_bf16(g);

    std::vector<float> wt, at, gin;
    for (int l = L - 1; l >= 0; --l) {
        size_t d = m->dims[l], u = m->dims[l + 1];
        if (l < L - 1) {
            // relu node of layer l: mask from the relu input; A > 0 <=> Z > 0.
            const auto& a = m->act[l + 1];
            for (size_t i = 0; i < n * u; ++i) g[i] = g[i] * (a[i] > 0.0f ? 1.0f : 0.0f);
            if (round_delta) round_bf16(g);
        }
        // add node: adjoint of b.
        reduce_rows(g.data(), m->db[l].data(), n, u);
        // matmul node: first g * W^T, then x^T * g.
        bool need_dx = (l > 0) || input_grad;
        if (need_dx) {
            wt.resize(u * d);
            transpose(gemm_weights(m, l), wt.data(), d, u);
            gin.resize(n * d);
            matmul(g.data(), wt.data(), gin.data(), n, u, d, threads);
        }
        at.resize(d * n);
        transpose(m->act[l].data(), at.data(), n, d);
        matmul(at.data(), g.data(), m->dW[l].data(), d, n, u, threads);
        if (l > 0) g.swap(gin);
    }

    if (optimizer == OR_OPT_ADAM) {
        m->t += 1;
        if (m->mW.empty()) {
            for (int l = 0; l < L; ++l) {
                m->mW.emplace_back(m->W[l].size(), 0.0f);
                m->vW.emplace_back(m->W[l].size(), 0.0f);
                m->mb.emplace_back(m->b[l].size(), 0.0f);
                m->vb.emplace_back(m->b[l].size(), 0.0f);
            }
        }
        for (int l = 0; l < L; ++l) {
            or_adam_update(m->W[l].data(), m->mW[l].data(), m->vW[l].data(), m->dW[l].data(),
                           m->W[l].size(), lr, 0.9f, 0.999f, 1e-8f, m->t);
            or_adam_update(m->b[l].data(), m->mb[l].data(), m->vb[l].data(), m->db[l].data(),
                           m->b[l].size(), lr, 0.9f, 0.999f, 1e-8f, m->t);
        }
    } else if (optimizer == OR_OPT_SGD) {
        for (int l = 0; l < L; ++l) {
            or_sgd_update(m->W[l].data(), nullptr, m->dW[l].data(), m->W[l].size(), lr, 0.0f);
            or_sgd_update(m->b[l].data(), nullptr, m->db[l].data(), m->b[l].size(), lr, 0.0f);
        }
    }
    return loss;
}

}  // extern "C"
