// host_util.hpp -- status codes and the thread-local error message behind
// q3_last_error().
#pragma once

#include <cuda_runtime.h>

#include <cstdio>
#include <exception>
#include <new>
#include <string>

#include "../../include/q3_sm100a.h"

namespace q3 {

void set_error(const std::string& msg);

struct Failure {
    int status;
};

inline int fail(int status, const std::string& msg) {
    set_error(msg);
    return status;
}

#define Q3_CUDA(call)                                                                                         \
    do {                                                                                                      \
        cudaError_t e_ = (call);                                                                              \
        if (e_ != cudaSuccess) {                                                                              \
            ::q3::set_error(std::string(#call) + ": " + cudaGetErrorString(e_));                              \
            return Q3_ERR_CUDA;                                                                               \
        }                                                                                                     \
    } while (0)

// Engine facts for host code outside engine.cu.
bool engine_tied(const q3_engine* e);
size_t engine_layers(const q3_engine* e);
size_t engine_capacity(const q3_engine* e);

#define Q3_CHECK(cond, msg)                                \
    do {                                                   \
        if (!(cond)) return ::q3::fail(Q3_ERR_INVALID, msg); \
    } while (0)

#define Q3_TRY_STATUS(x)               \
    do {                               \
        const int rc_ = (x);           \
        if (rc_ != Q3_OK) return rc_;  \
    } while (0)

// Runs the body of a C entry point whose host work allocates in proportion to
// its input (files, text): no C++ exception crosses the C ABI.  A failed host
// allocation becomes Q3_ERR_OOM, any other exception Q3_ERR_INVALID with its
// message.
template <class F>
int guarded(const char* fn, F&& body) noexcept {
    try {
        return body();
    } catch (const std::bad_alloc&) {
        return fail(Q3_ERR_OOM, std::string(fn) + ": host allocation failed");
    } catch (const std::exception& ex) {
        return fail(Q3_ERR_INVALID, std::string(fn) + ": " + ex.what());
    } catch (...) {
        return fail(Q3_ERR_INVALID, std::string(fn) + ": unexpected exception");
    }
}

}  // namespace q3
