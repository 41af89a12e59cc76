// internal.h -- host-side helpers shared by the translation units of libttl_moe.
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "ttl_moe.h"

struct ttl_moe;

namespace ttl {

// Records `message` as the last error of `handle` (or of the calling thread
// when handle is null) and returns `code`.
int fail(ttl_moe *handle, int code, const std::string &message);
std::string &thread_error();
const char *handle_error(const ttl_moe *handle);

// True when `p` is device memory (or managed memory) of some GPU.
bool is_device_pointer(const void *p);

} // namespace ttl

#define TTL_TRY_CUDA(handle, expr)                                                                     \
    do {                                                                                               \
        const cudaError_t ttl_err_ = (expr);                                                           \
        if (ttl_err_ != cudaSuccess) {                                                                 \
            return ttl::fail((handle), TTL_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(ttl_err_)); \
        }                                                                                              \
    } while (0)
