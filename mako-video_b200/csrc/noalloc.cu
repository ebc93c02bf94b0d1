// h3k_sparse_attention_noalloc: the block-sparse attention (cube selection, pass lists and the sparse flash kernel)
// without any device allocation. Some callers cannot call cudaMalloc around every attention call: a serving stack
// that has reserved nearly all of the GPU's memory for its own pool (an extra cudaMalloc can fail), or a caller whose
// other streams must not stall (cudaMalloc and cudaFree synchronise the whole device). For them the scratch the
// sparse path needs (cube means of q and k, cube scores, selections, pass lists) lives in one fixed array in this
// library's device memory instead.
//
// The array below is held by every GPU that loads the library until the process exits. Every call shares it and it
// keeps the last call's contents: calls whose work overlaps on the GPU (two streams, or two host threads) race on it.
// Its device address is looked up on the first call made in each CUDA context (normally once per device: the
// device's primary context); make that first call before any stream capture. The lookup is keyed by the context's
// process-unique id, so a context torn down and created again (cudaDeviceReset) gets a fresh lookup instead of the
// old context's address.
#include "h3_c.h"

#include "attention.cuh"
#include "common.hpp"
#include "sparse.cuh"

#include <functional>
#include <mutex>
#include <string>

namespace h3 {
int run_guarded(const std::function<void()>& f); // capi.cpp: the status codes and message of every entry point
} // namespace h3

namespace {

// The no-allocation scratch: 16 MiB (e.g. 5 heads over the 528 cubes of a 768p grid, one rank of eight, need ~10 MB).
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
struct ScratchAddr {
    unsigned long long context_id = 0; // the context the address belongs to (0: none looked up yet)
    void* addr = nullptr;
};
ScratchAddr g_scratch[kMaxDevices];

using CtxGetCurrent = CUresult (*)(CUcontext*);
using CtxGetId = CUresult (*)(CUcontext, unsigned long long*);

template <class Fn>
Fn driver_fn(const char* name)
{
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    H3_CUDA(cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !p)
        throw h3::CudaError(std::string(name) + " is not available from the driver");
    return reinterpret_cast<Fn>(p);
}

// The process-unique id of the current context (the driver never hands the same id to two contexts, unlike the
// context handle, which a re-created context may reuse).
unsigned long long current_context_id()
{
    static const CtxGetCurrent get_current = driver_fn<CtxGetCurrent>("cuCtxGetCurrent");
    static const CtxGetId get_id = driver_fn<CtxGetId>("cuCtxGetId");
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
        throw h3::CudaError("no-allocation scratch: no current CUDA context");
    return id;
}

// The scratch's device address in the current context (cudaGetSymbolAddress once per context). In host code the
// array's name is only a stand-in, so kernels are always given this address.
void* scratch_for_current_device()
{
    int dev = 0;
    H3_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices)
        throw h3::CudaError("no-allocation scratch: device index out of range");
    H3_CUDA(cudaSetDevice(dev)); // makes the device's primary context current if nothing has yet
    const unsigned long long ctx = current_context_id();
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    ScratchAddr& e = g_scratch[dev];
    if (e.context_id != ctx || !e.addr) {
        void* p = nullptr;
        const cudaError_t rc = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (rc != cudaSuccess || !p)
            throw h3::CudaError(std::string("no-allocation scratch: cudaGetSymbolAddress failed: ") + cudaGetErrorString(rc));
        e.context_id = ctx;
        e.addr = p;
    }
    return e.addr;
}

size_t round256(size_t n) { return (n + 255) & ~size_t(255); }

} // namespace

extern "C" int h3k_sparse_attention_noalloc(const void* q, const void* k, const void* v, int64_t row_stride, int32_t heads,
                                            const h3k_cube_grid* g, float ratio, int32_t local, void* out, int64_t out_row_stride,
                                            void* stream)
{
    return h3::run_guarded([&] {
        if (!q || !k || !v || !out || !g || heads <= 0)
            throw std::invalid_argument("h3k_sparse_attention_noalloc: null argument or no heads");
        if (g->frames <= 0 || g->ph <= 0 || g->pw <= 0 || g->dense_rows < 0)
            throw std::invalid_argument("h3k_sparse_attention_noalloc: bad cube grid");
        for (const void* ptr : {q, k, v, static_cast<const void*>(out)})
            if (!h3::device_accessible(ptr))
                throw std::invalid_argument("h3k_sparse_attention_noalloc: a pointer argument is host memory the GPU cannot access");
        h3::CubeGrid c;
        c.dense_rows = g->dense_rows, c.frames = g->frames, c.ph = g->ph, c.pw = g->pw;
        c.nct = (c.frames + 3) / 4, c.ncy = (c.ph + 3) / 4, c.ncx = (c.pw + 3) / 4;
        h3::SparseBuffers b;
        h3::sparse_sizes(c, ratio, local, b.kcap, b.q_tiles, b.max_blocks);
        const size_t nc = size_t(c.cubes()), H = size_t(heads);
        const size_t sizes[8] = {H * nc * 128 * 4, H * nc * 128 * 4, H * nc * nc * 4, H * nc * b.kcap * 4, H * nc * 4,
                                 H * b.q_tiles * b.max_blocks * 16, H * b.q_tiles * 4, size_t(b.q_tiles) * 16};
        size_t need = 0;
        for (size_t s : sizes)
            need += round256(s);
        if (need > kNoAllocScratchBytes)
            throw std::invalid_argument("h3k_sparse_attention_noalloc: this grid and head count need " + std::to_string(need) +
                                        " bytes of scratch; the fixed scratch holds " + std::to_string(kNoAllocScratchBytes) +
                                        " (use h3k_sparse_attention, or fewer heads per call)");
        uint8_t* base = static_cast<uint8_t*>(scratch_for_current_device());
        uint8_t* p = base;
        auto take = [&](size_t n) {
            uint8_t* r = p;
            p += round256(n);
            return r;
        };
        b.mq = reinterpret_cast<float*>(take(sizes[0]));
        b.mk = reinterpret_cast<float*>(take(sizes[1]));
        b.scores = reinterpret_cast<float*>(take(sizes[2]));
        b.sel = reinterpret_cast<int32_t*>(take(sizes[3]));
        b.nsel = reinterpret_cast<int32_t*>(take(sizes[4]));
        b.blocks = reinterpret_cast<int4*>(take(sizes[5]));
        b.nblocks = reinterpret_cast<int32_t*>(take(sizes[6]));
        b.q_rows = reinterpret_cast<int4*>(take(sizes[7]));
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        // Every buffer is written before it is read within one call; clearing the part in use anyway keeps a call
        // from ever seeing the previous call's selections.
        H3_CUDA(cudaMemsetAsync(base, 0, need, s));
        h3::AttnParams a;
        a.q = q, a.k = k, a.v = v, a.row_stride = row_stride, a.heads = heads, a.rows = c.dense_rows + c.frames * c.ph * c.pw;
        a.out = out, a.out_row_stride = out_row_stride;
        h3::sparse_attention(a, c, ratio, local, b, s);
    });
}
