// A device allocation owned by one object (the model's weights and activation buffers): grown on demand, zeroed
// when (re)allocated, freed on destruction.
#pragma once
#include "common.hpp"

#include <cuda_runtime.h>

#include <cstddef>

namespace h3 {

struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : p(o.p), bytes(o.bytes) { o.p = nullptr, o.bytes = 0; }
    DevBuf& operator=(DevBuf&& o) noexcept
    {
        if (this != &o) {
            release();
            p = o.p, bytes = o.bytes;
            o.p = nullptr, o.bytes = 0;
        }
        return *this;
    }
    ~DevBuf() { release(); }
    void release()
    {
        if (p)
            cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    void ensure(size_t n)
    {
        if (n <= bytes)
            return;
        release();
        H3_CUDA(cudaMalloc(&p, n));
        // The legacy-stream memset is not ordered with the model's non-blocking stream: finish it before anything is
        // queued there (growth is rare: the first step of a layout or of more noise levels).
        H3_CUDA(cudaMemset(p, 0, n));
        H3_CUDA(cudaDeviceSynchronize());
        bytes = n;
    }
    template <class T>
    T* as() const
    {
        return static_cast<T*>(p);
    }
};

} // namespace h3
