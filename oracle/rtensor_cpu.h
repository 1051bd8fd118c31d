/*
 * CPU oracle: a C++ restatement of rtensor's CPU backend (the Rust crate
 * `rtensor` in MMMejias39/RGPU, crates/rtensor/src).
 *
 * THIS IS TEST INFRASTRUCTURE.  It is the checker that the CUDA path is
 * compared against, and the timed CPU baseline.  Nothing in the product
 * library (rgpu_b200/librtgpu.so) links, loads or calls it.
 *
 * Every routine follows the loop order and the f32 rounding sequence of the
 * reference function it cites, so that results are bit-identical to what the
 * Rust code computes on the same host (the file is compiled with
 * -ffp-contract=off: Rust never fuses a*b+c into an FMA).
 *
 * Parity pin: the reference cannot be compiled here (no Rust toolchain), so
 * the restatement is pinned on the known-answer tests of
 * crates/rtensor/tests/autodiff.rs (matmul 2x3*3x2 = [58,64,139,154],
 * broadcast add, reduce_to, softmax of logits 100, transpose involution,
 * gradient accumulation [3,5,7]) and on its central-difference gradient
 * checks, all re-run in tests/test_oracle.py.
 */
#ifndef RTENSOR_CPU_ORACLE_H
#define RTENSOR_CPU_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- Rng: xorshift64* (crates/rtensor/src/rng.rs:1-49) ------------------ */
uint64_t or_rng_seed(uint64_t seed);                       /* Rng::new        rng.rs:8-10  */
void or_rng_uniform(uint64_t* state, float* out, size_t n); /* Rng::uniform    rng.rs:22-24 */
void or_rng_range(uint64_t* state, float lo, float hi, float* out, size_t n); /* rng.rs:27-29 */
void or_rng_normal(uint64_t* state, float* out, size_t n);  /* Rng::normal     rng.rs:32-36 */
void or_rng_below(uint64_t* state, uint64_t n, uint32_t* out, size_t count); /* rng.rs:38-40 */

/* ---- Tensor kernels (crates/rtensor/src/tensor.rs) ---------------------- */
/* C[m,n] = A[m,k] B[k,n]: ikj axpy order with zero-skip, blocked JC=256/PC=128
 * above k*n > 32768 (tensor.rs:318-373). */
void or_matmul(const float* a, const float* b, float* c, size_t m, size_t k, size_t n, int threads);
/* out[c,r] = a[r,c]^T, 32x32 blocks (tensor.rs:132-155). */
void or_transpose(const float* a, float* out, size_t r, size_t c);
/* out[1,m] = 1_n^T g: row-sequential accumulation (tensor.rs:410-418). */
void or_reduce_rows(const float* g, float* out, size_t n, size_t m);
/* out[r,c] = softmax of each row, max-stabilised (tensor.rs:455-472). */
void or_softmax_rows(const float* z, float* out, size_t r, size_t c);
/* Softmax cross-entropy over one-hot targets (losses.rs:99-115, the
 * `softmax_cross_entropy` node).  Returns the loss value; when `dlogits` is
 * non-null writes the node's adjoint (P - Y) * (g/n) with g = 1. */
float or_softmax_xent(const float* logits, const float* onehot, size_t n, size_t c, float* dlogits);
/* losses::one_hot (losses.rs:169-175). */
void or_one_hot(const uint32_t* labels, size_t n, size_t classes, float* out);

/* ---- Dense/Sequential ReLU MLP trained through the tape ------------------ */
/* Layers l = 0..L-1 with W_l[dims[l], dims[l+1]], b_l[1, dims[l+1]].
 * Hidden layers use ReLU, the last one is linear (nn.rs:143-149), the loss is
 * softmax cross-entropy over one-hot labels. */
typedef struct or_mlp or_mlp;

or_mlp* or_mlp_new(int n_layers, const size_t* dims);
void or_mlp_free(or_mlp* m);
/* Copy W_l / b_l in (row-major). */
void or_mlp_set(or_mlp* m, int layer, const float* w, const float* b);
void or_mlp_get(const or_mlp* m, int layer, float* w, float* b);
/* Gradients of the last step (Grads::of for W_l / b_l). */
void or_mlp_get_grads(const or_mlp* m, int layer, float* dw, float* db);
/* Logits of the last forward. */
void or_mlp_get_logits(const or_mlp* m, float* out);

/* Glorot-uniform init of Dense::new (nn.rs:122-130) from an Rng state,
 * layer by layer in order; b = 0. */
void or_mlp_init_glorot(or_mlp* m, uint64_t* rng_state);
/* Kaiming-uniform init U(-sqrt(6/fan_in), +sqrt(6/fan_in)) through the same
 * Rng::range draw order; b = 0. */
void or_mlp_init_kaiming(or_mlp* m, uint64_t* rng_state);

enum { OR_OPT_NONE = 0, OR_OPT_SGD = 1, OR_OPT_ADAM = 2 };

/* One training step exactly as the reference's CPU loop does it:
 *   Tape::new, constant(x), Sequential::forward, softmax_cross_entropy,
 *   Var::backward (tape.rs:187-229), Optimizer::step (optim.rs).
 * Returns the loss value.  `threads` > 1 splits the row loop of each matmul
 * across host threads (every output element keeps its summation order, so
 * results are identical for any thread count).  `input_grad` = 1 also
 * computes the adjoint of x, which the tape always does (ops.rs:128). */
float or_mlp_train_step(or_mlp* m, const float* x, const uint32_t* labels, size_t n,
                        int optimizer, float lr, int threads, int input_grad);
/* bf16 rounding emulation (NOT part of the reference algorithm; test-only).
 * Each flag rounds to bf16 (nearest even) at one storage point of the bf16
 * GPU plan; arithmetic between those points stays f32, in the reference's
 * loop order:
 *   OR_ROUND_X      the input x;
 *   OR_ROUND_W      the weights the GEMMs read (the optimiser still updates
 *                   the f32 masters);
 *   OR_ROUND_ACT    every hidden activation after bias+ReLU, wherever it is
 *                   read (next layer's forward, dW, ReLU mask);
 *   OR_ROUND_DELTA  every adjoint delta_l before it feeds a GEMM or the bias
 *                   reduction;
 *   OR_SPLIT_ACT    every hidden activation a is rounded to hi = bf16(a) and,
 *                   where it feeds another hidden layer, that layer's forward
 *                   reads hi + bf16(a - hi); the dW product, the ReLU mask
 *                   and the output layer's forward read hi (the
 *                   split-activation plan; overrides OR_ROUND_ACT).
 * With no flag set the oracle is the plain reference. */
enum { OR_ROUND_X = 1, OR_ROUND_W = 2, OR_ROUND_ACT = 4, OR_ROUND_DELTA = 8, OR_SPLIT_ACT = 16 };
void or_mlp_set_rounding(or_mlp* m, int flags);
/* Shorthand: on = OR_ROUND_X | OR_ROUND_W | OR_ROUND_ACT | OR_ROUND_DELTA
 * (the plan with single-bf16 activations), off = plain reference. */
void or_mlp_set_bf16_emulation(or_mlp* m, int on);

/* Forward only (Sequential::predict, nn.rs:184-188); returns the loss of the
 * logits against the labels when labels != NULL. */
float or_mlp_forward(or_mlp* m, const float* x, const uint32_t* labels, size_t n, int threads);

/* Adam (optim.rs:142-199) and SGD (optim.rs:64-115) on a single flat buffer,
 * exposed for unit parity of the update kernels.  `t` is the step number
 * after the increment (1 on the first step). */
void or_adam_update(float* theta, float* m, float* v, const float* g, size_t n,
                    float lr, float beta1, float beta2, float eps, int t);
void or_sgd_update(float* theta, float* vel, const float* g, size_t n, float lr, float momentum);

#ifdef __cplusplus
}
#endif
#endif
