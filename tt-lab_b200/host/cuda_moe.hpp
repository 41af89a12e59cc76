// cuda_moe.hpp -- C++ face of the CUDA MoE backend for tt-lab's host code.
//
// tt-lab reports failures as std::runtime_error and main() prints
// "error: <message>" (src/main.cpp:414-417); this header turns the C ABI's
// status codes into exactly that, so the backend drops into GptOssModel and the
// requant path with the reference's error behaviour.  Header-only, no CUDA
// headers needed by the includer.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "ttl_moe.h"

namespace ttl {

inline void check(int rc, const ttl_moe *handle = nullptr) {
    if (rc != TTL_OK) {
        throw std::runtime_error(std::string("cuda moe: ") + ttl_moe_last_error(handle));
    }
}

// Owns one ttl_moe handle (one GPU; one expert-parallel rank).
class CudaMoe {
  public:
    explicit CudaMoe(const ttl_moe_config &config) {
        check(ttl_moe_create(&config, &handle_));
    }
    ~CudaMoe() {
        ttl_moe_destroy(handle_);
    }
    CudaMoe(const CudaMoe &) = delete;
    CudaMoe &operator=(const CudaMoe &) = delete;

    // Binds one layer's GGUF MoE tensors (src/model.cpp:157-169 names).
    void upload_layer(int layer, const float *router_w, const float *router_b, const void *gate_w,
                      const float *gate_b, const void *up_w, const float *up_b, const void *down_w,
                      const float *down_b) {
        check(ttl_moe_upload_layer(handle_, layer, router_w, router_b, gate_w, gate_b, up_w, up_b, down_w, down_b),
              handle_);
    }
    void upload_norm(int layer, const float *norm_w) {
        check(ttl_moe_upload_norm(handle_, layer, norm_w), handle_);
    }
    // GptOssModel::moe replacement (host buffers, blocking).
    void moe(int layer, const float *input, float *output, int32_t *top4_idx = nullptr, float *top4_w = nullptr) {
        check(ttl_moe_decode(handle_, layer, input, output, top4_idx, top4_w), handle_);
    }
    // GptOssModel::moe_batch replacement (host buffers, blocking).
    void moe_batch(int layer, const float *input, float *output, size_t count, int32_t *top4_idx = nullptr,
                   float *top4_w = nullptr) {
        check(ttl_moe_prefill(handle_, layer, input, count, output, top4_idx, top4_w), handle_);
    }
    // RMSNorm -> MoE -> residual over layers [begin, end) for `tokens` tokens.
    void forward(int begin, int end, const float *x, float *y, size_t tokens) {
        check(ttl_moe_forward(handle_, begin, end, x, y, tokens), handle_);
    }
    ttl_moe *get() const {
        return handle_;
    }

  private:
    ttl_moe *handle_ = nullptr;
};

} // namespace ttl
