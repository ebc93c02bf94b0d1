// Host helpers: tensor-map encoding through the driver entry point, the device error word, the SM count.
#include "common.hpp"
#include "ptx.cuh"

#include <mutex>

namespace h3 {

__device__ uint32_t g_device_error = 0;

namespace {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                 const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn()
{
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        H3_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !p)
            throw CudaError("cuTensorMapEncodeTiled is not available from the driver");
        fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

} // namespace

CUtensorMap make_tmap(CUtensorMapDataType type, int rank, const void* base, const uint64_t* dims, const uint64_t* strides_bytes,
                      const uint32_t* box, bool swizzle128)
{
    CUtensorMap m;
    cuuint64_t d[5];
    cuuint64_t st[4];
    cuuint32_t b[5], es[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        es[i] = 1;
        if (i + 1 < rank)
            st[i] = strides_bytes[i];
    }
    if (reinterpret_cast<uintptr_t>(base) % 16)
        throw CudaError("tensor map: base address not 16-byte aligned");
    const CUresult r = encode_fn()(&m, type, cuuint32_t(rank), const_cast<void*>(base), d, st, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                   swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        throw CudaError("cuTensorMapEncodeTiled failed with code " + std::to_string(int(r)));
    return m;
}

uint32_t take_device_error(cudaStream_t s)
{
    uint32_t v = 0, zero = 0;
    H3_CUDA(cudaMemcpyFromSymbolAsync(&v, g_device_error, sizeof(v), 0, cudaMemcpyDeviceToHost, s));
    H3_CUDA(cudaStreamSynchronize(s));
    if (v)
        H3_CUDA(cudaMemcpyToSymbolAsync(g_device_error, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s));
    return v;
}

bool device_accessible(const void* p)
{
    if (!p)
        return true;
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type != cudaMemoryTypeUnregistered && a.devicePointer != nullptr;
}

uint64_t device_bit()
{
    int dev = 0;
    H3_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev > 63)
        throw CudaError("device index past 63");
    return uint64_t(1) << dev;
}

int num_sms()
{
    int dev = 0, n = 0;
    H3_CUDA(cudaGetDevice(&dev));
    H3_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    return n;
}

} // namespace h3
