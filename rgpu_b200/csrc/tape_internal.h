// Shared internals of the GPU autodiff tape (tape.cu: leaves, matmul, add,
// ReLU, softmax-CE, backward, optimisers; tape_ops.cu: the remaining
// elementwise, reduction and loss ops).
#pragma once

#include <functional>
#include <unordered_map>
#include <vector>

#include "internal.h"

namespace rt {
int run_gemm(rt_ctx* ctx, GemmDesc g, cudaStream_t stream, size_t ws_bytes);

int launch_axpy_inplace(rt_ctx* ctx, float* dst, int64_t ldd, const float* src, int64_t lds, int64_t rows,
                        int64_t cols, cudaStream_t st);
int launch_mean_rows(rt_ctx* ctx, const float* rows, int64_t n, float* out, cudaStream_t st);

namespace tp {

inline int64_t ld_for(int64_t cols) { return cols <= 4 ? 4 : (cols + 3) / 4 * 4; }

// A device f32 matrix owned by a tape (or borrowed from a parameter).
struct Buf {
    float* p = nullptr;
    int64_t rows = 0, cols = 0, ld = 0;
};

struct Node {
    std::vector<int> parents;
    // Given the node's adjoint, adds each parent's contribution (via acc).
    std::function<int(const Buf& g)> backward;
    Buf value;
};

}  // namespace tp
}  // namespace rt

struct rt_param {
    rt_ctx* ctx = nullptr;
    rt::tp::Buf value;
    uint64_t id = 0;
};

struct rt_var {
    rt_tape* tape = nullptr;
    int idx = 0;
};

struct rt_tape {
    using Buf = rt::tp::Buf;
    rt_ctx* ctx = nullptr;
    std::vector<rt::tp::Node> nodes;
    std::vector<rt_var*> vars;
    std::unordered_map<uint64_t, int> param_nodes;
    std::vector<Buf> grads;   // adjoint per node after backward (p == nullptr: none)
    std::vector<void*> owned; // stream-ordered allocations to release
    bool backward_done = false;

    int alloc(Buf& b, int64_t rows, int64_t cols) {
        b.rows = rows;
        b.cols = cols;
        b.ld = rt::tp::ld_for(cols);
        size_t bytes = (size_t)(rows > 0 ? rows : 1) * (size_t)b.ld * 4;
        RT_CUDA(cudaMallocAsync((void**)&b.p, bytes, ctx->stream));
        owned.push_back(b.p);
        RT_CUDA(cudaMemsetAsync(b.p, 0, bytes, ctx->stream));
        return RT_OK;
    }

    rt_var* push(std::vector<int> parents, std::function<int(const Buf&)> bw, const Buf& value) {
        rt::tp::Node n;
        n.parents = std::move(parents);
        n.backward = std::move(bw);
        n.value = value;
        nodes.push_back(std::move(n));
        rt_var* v = new rt_var;
        v->tape = this;
        v->idx = (int)nodes.size() - 1;
        vars.push_back(v);
        return v;
    }

    // grads[i] += g   (allocates the adjoint on first contribution)
    int accumulate(int i, const Buf& g) {
        Buf& dst = grads[i];
        if (!dst.p) {
            RT_TRY(alloc(dst, g.rows, g.cols));
            RT_CUDA(cudaMemcpy2DAsync(dst.p, dst.ld * 4, g.p, g.ld * 4, g.cols * 4, g.rows, cudaMemcpyDeviceToDevice,
                                      ctx->stream));
            return RT_OK;
        }
        return rt::launch_axpy_inplace(ctx, dst.p, dst.ld, g.p, g.ld, g.rows, g.cols, ctx->stream);
    }
};

namespace rt {
namespace tp {
inline int check_var(const rt_var* v) {
    RT_CHECK(v && v->tape && v->idx >= 0 && v->idx < (int)v->tape->nodes.size(), "invalid variable");
    return RT_OK;
}
}  // namespace tp
}  // namespace rt
