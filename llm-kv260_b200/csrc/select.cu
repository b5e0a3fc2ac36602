// Greedy token selection on the device: the first index of the largest value,
// as the runtime's scan does (board/tp/tp_llama.cpp:879-882: `if (y[i] >
// y[best]) best = i`, strict >, so the lowest index wins a tie). The scan's
// NaN behaviour is kept too: a NaN at index 0 is never beaten, a NaN anywhere
// else never wins.
//
// Two kernels: CTAs reduce slices to (value, index) candidates in a scratch
// array, then one CTA reduces the candidates. The pair order is
// (value descending, index ascending), the order sample_token sorts its
// candidates by (tp_llama.cpp:924).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "../../include/b200_engine.h"
#include "common.cuh"

namespace b200 {

namespace {

constexpr int kSelThreads = 512;

struct Cand {
    float v;
    int i;
};

// a before b in (value desc, index asc); NaN values sort last (index 0 is
// handled before the reduction).
__device__ __forceinline__ bool better(const Cand &a, const Cand &b) {
    if (isnan(b.v)) return !isnan(a.v) || a.i < b.i;
    if (isnan(a.v)) return false;
    return a.v > b.v || (a.v == b.v && a.i < b.i);
}

__device__ __forceinline__ Cand block_best(Cand c) {
    __shared__ Cand red[kSelThreads / 32];
    for (int off = 16; off > 0; off >>= 1) {
        Cand o;
        o.v = __shfl_down_sync(kFullMask, c.v, off);
        o.i = __shfl_down_sync(kFullMask, c.i, off);
        if (better(o, c)) c = o;
    }
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (lane == 0) red[warp] = c;
    __syncthreads();
    if (warp == 0) {
        c = lane < static_cast<int>(blockDim.x / 32) ? red[lane] : Cand{NAN, 0x7fffffff};
        for (int off = 16; off > 0; off >>= 1) {
            Cand o;
            o.v = __shfl_down_sync(kFullMask, c.v, off);
            o.i = __shfl_down_sync(kFullMask, c.i, off);
            if (better(o, c)) c = o;
        }
    }
    return c;
}

__global__ void __launch_bounds__(kSelThreads) argmax_partial_kernel(const float *__restrict__ y, int n,
                                                                     Cand *__restrict__ part) {
    pdl_launch_dependents();
    pdl_wait_prior_grid();
    Cand c{NAN, 0x7fffffff};
    for (int i = blockIdx.x * kSelThreads + threadIdx.x; i < n; i += gridDim.x * kSelThreads) {
        const Cand o{y[i], i};
        if (better(o, c)) c = o;
    }
    c = block_best(c);
    if (threadIdx.x == 0) part[blockIdx.x] = c;
}

__global__ void __launch_bounds__(kSelThreads) argmax_final_kernel(const float *__restrict__ y, const Cand *part,
                                                                   int nparts, int index_base, int *out_index,
                                                                   float *out_value) {
    pdl_launch_dependents();
    pdl_wait_prior_grid();
    Cand c{NAN, 0x7fffffff};
    for (int i = threadIdx.x; i < nparts; i += kSelThreads)
        if (better(part[i], c)) c = part[i];
    c = block_best(c);
    if (threadIdx.x == 0) {
        if (isnan(y[0]) || c.i == 0x7fffffff) c = Cand{y[0], 0};
        *out_index = c.i + index_base;
        *out_value = c.v;
    }
}

}  // namespace

int argmax_scratch_bytes() { return static_cast<int>(sizeof(Cand)) * kArgmaxMaxParts; }

int argmax_launch(const float *y, int n, int index_base, void *scratch, int *out_index, float *out_value,
                  cudaStream_t stream, bool pdl) {
    if (!y || n <= 0 || !scratch || !out_index || !out_value) return kErrInval;
    int parts = (n + kSelThreads * 4 - 1) / (kSelThreads * 4);
    const int sms = sm_count();
    if (sms > 0 && parts > sms) parts = sms;
    if (parts > kArgmaxMaxParts) parts = kArgmaxMaxParts;
    if (parts < 1) parts = 1;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg{};
    cfg.blockDim = dim3(kSelThreads);
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cfg.gridDim = dim3(parts);
    Cand *part = static_cast<Cand *>(scratch);
    if (cudaLaunchKernelEx(&cfg, argmax_partial_kernel, y, n, part) != cudaSuccess) return kErrCuda;
    cfg.gridDim = dim3(1);
    if (cudaLaunchKernelEx(&cfg, argmax_final_kernel, y, static_cast<const Cand *>(part), parts, index_base,
                           out_index, out_value) != cudaSuccess)
        return kErrCuda;
    return 0;
}

// ---------------------------------------------------------------------------
// The greedy pick for callers that cannot allocate device memory.
//
// b200_argmax_f32 needs an engine, and opening an engine calls cudaMalloc
// for its scratch. Some callers cannot do that: code that runs while a CUDA
// graph is being captured, a caller whose memory is handed out by its own
// pool or allocator (and must not see a second one), or a host that loads
// this library into a process where device allocation is forbidden after
// start-up. b200_argmax_f32_noalloc gives them the same pick with no
// allocation at all: its scratch (one (value, index) candidate per CTA of
// the first pass, 1024 of them, 8 KB) is the file-scope array below, which
// every GPU that loads the library holds until the process exits.
//
// In host code `g_noalloc_cand` is only a stand-in for the symbol, not a
// device address: passing it to a kernel would fault, or where the GPU can
// reach host memory, silently use the wrong memory. So the first call on a
// device, with that device current, asks cudaGetSymbolAddress for the real
// address and keeps it for that device; later calls reuse it. Because of
// that look-up, make the first call on each device before any stream
// capture.
//
// Every call shares the one array and it keeps the last call's contents.
// Nothing in it has to start at zero: a call writes every candidate it
// reads. Calls whose kernels overlap on the GPU (different streams, or
// different host threads) race on the array; run them one at a time.
// ---------------------------------------------------------------------------

namespace {

constexpr int kNoAllocParts = kArgmaxMaxParts;  // candidate slots
constexpr int kNoAllocMaxN = 1 << 25;           // largest y accepted: 33,554,432 floats

static __device__ __align__(256) Cand g_noalloc_cand[kNoAllocParts];

std::mutex g_noalloc_mu;
void *g_noalloc_ptr[64] = {};

}  // namespace

}  // namespace b200

extern "C" int b200_argmax_f32_noalloc(uint64_t y, int n, int index_base, uint64_t out, void *stream) {
    using namespace b200;
    if (!y || !out || y % 4 || out % 4)
        return report_error(kErrInval, "argmax (no-alloc): y and out must be non-null and 4-byte aligned");
    if (n <= 0) return report_error(kErrInval, "argmax (no-alloc): n must be positive");
    if (n > kNoAllocMaxN) {
        char msg[160];
        snprintf(msg, sizeof msg, "argmax (no-alloc): n = %d is above the limit of %d elements", n, kNoAllocMaxN);
        return report_error(kErrInval, msg);
    }
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return report_error(kErrNoDev, "argmax (no-alloc): no usable current CUDA device");
    void *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!g_noalloc_ptr[dev]) {
            void *p = nullptr;
            const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_cand);
            if (err != cudaSuccess || !p) {
                char msg[200];
                snprintf(msg, sizeof msg, "argmax (no-alloc): cudaGetSymbolAddress failed on device %d: %s", dev,
                         cudaGetErrorString(err));
                return report_error(kErrCuda, msg);
            }
            g_noalloc_ptr[dev] = p;
        }
        scratch = g_noalloc_ptr[dev];
    }
    int *oi = reinterpret_cast<int *>(out);
    if (argmax_launch(reinterpret_cast<const float *>(y), n, index_base, scratch, oi, reinterpret_cast<float *>(oi + 1),
                      static_cast<cudaStream_t>(stream), false)) {
        char msg[200];
        snprintf(msg, sizeof msg, "argmax (no-alloc): launch failed: %s", cudaGetErrorString(cudaGetLastError()));
        return report_error(kErrCuda, msg);
    }
    return 0;
}
