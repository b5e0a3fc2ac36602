// Tensor-parallel exchange over NVLink peer memory (include/b200_comm.h):
// the rank-ordered all-reduce of board/tp/tp_llama.cpp:504-525, the
// all-gather of :482-490 and the greedy candidate exchange of :894-925.
//
// Window. Every rank cudaMallocs one window and exports it by CUDA IPC; every
// peer maps it. Layout:
//     [0, 2*R*G*256*8)       all-reduce receive words, [slot][source rank][element]
//     [ag, ag + 2*256*R)     all-gather data, two slots of R ranks x 256 B
//     [agflags, +R*8)        all-gather arrival flags: [source rank]
//     [counters, +(G+1)*8)   this rank's epoch per chunk CTA, + the all-gather's
//     [status, +4)           value 2: a wait for a peer ran out
// Chunks are fixed at 256 floats, so CTA c of every call always owns the same
// elements; its epoch e (a device counter, so graphs replay correctly) picks
// slot e & 1.
//
// All-reduce, per element, on every rank (one thread per element):
//   1. push the 8-byte word {value bits, epoch} into slot e & 1, row [this
//      rank], of every rank's window (its own included) -- one store each,
//      no fence: an 8-byte store lands whole, so a reader that sees the
//      epoch sees the value (the low-latency protocol NCCL calls LL);
//   2. spin (bounded) on the own window until every rank's word for this
//      element carries epoch e;
//   3. sum in rank order, s = p0; s = s + p_r, r = 1..n-1 --
//      tp_llama.cpp:515-521 exactly, so every rank gets the same bits -- and
//      write the result in place.
// The reference does a reduce-scatter then an all-gather (two TCP rounds);
// summing every element in the same rank order makes the one-shot exchange
// here produce the same bits. Two slots suffice: a rank writes slot s at
// epoch e+2 only after it saw every peer's epoch-(e+1) words, and a peer
// writes those only after its epoch-e kernel (which read slot s) finished.
// No TMA and no multicast: plain peer stores and local loads.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "../../include/b200_comm.h"
#include "common.cuh"
#include "decode.h"

namespace b200 {

namespace {

constexpr int kMaxRanks = 8;
constexpr int kChunk = 256;           // floats per all-reduce CTA
constexpr int kCommThreads = 256;
constexpr int kAgSlotBytes = 256;     // per rank per slot
constexpr uint64_t kPeerTimeoutNs = 1000000000ull;  // 1 s

struct CommParams {
    uint8_t *win[kMaxRanks];  // every rank's window as mapped in this process (own at [rank])
    int rank, nranks;
    int gmax;                 // all-reduce chunk CTAs the window has flags for
    uint64_t slot_words;      // words per (slot, source rank): gmax * 256
    uint64_t off_ag, off_agflags, off_counters, off_status;
};

__device__ __forceinline__ void st_word(uint64_t *p, uint64_t w) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ uint64_t ld_word(const uint64_t *p) {
    uint64_t w;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

__device__ __forceinline__ void st_release_sys(uint64_t *p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Bounded wait until *flag >= e. Returns false on timeout (and flags status).
__device__ __forceinline__ bool wait_flag(const uint64_t *flag, uint64_t e, unsigned *status) {
    if (ld_acquire_sys(flag) >= e) return true;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(flag) < e) {
        if (globaltimer_ns() - t0 > kPeerTimeoutNs) {
            atomicOr(status, kStatusPeerTimeout);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

__global__ void __launch_bounds__(kCommThreads) allreduce_kernel(const __grid_constant__ CommParams p, float *v,
                                                                 int len) {
    pdl_launch_dependents();
    pdl_wait_prior_grid();
    __shared__ uint64_t s_e;
    const int t = threadIdx.x, c = blockIdx.x;
    const int i = c * kChunk + t;
    uint8_t *own = p.win[p.rank];
    unsigned *status = reinterpret_cast<unsigned *>(own + p.off_status);
    if (t == 0) {
        uint64_t *ctr = reinterpret_cast<uint64_t *>(own + p.off_counters) + c;
        const uint64_t e = *ctr + 1;
        *ctr = e;
        s_e = e;
    }
    __syncthreads();
    const uint32_t e = static_cast<uint32_t>(s_e);
    if (i >= len) return;
    const uint64_t slot = (e & 1) * kMaxRanks * p.slot_words;
    const float mine = v[i];
    const uint64_t word = (static_cast<uint64_t>(e) << 32) | __float_as_uint(mine);
    for (int r = 0; r < p.nranks; ++r)
        st_word(reinterpret_cast<uint64_t *>(p.win[r]) + slot + p.rank * p.slot_words + i, word);
    const uint64_t *rx = reinterpret_cast<const uint64_t *>(own) + slot + i;
    float val[kMaxRanks];
    unsigned pending = (1u << p.nranks) - 1;
    const uint64_t t0 = globaltimer_ns();
    for (unsigned spins = 0; pending; ++spins) {
        for (int r = 0; r < p.nranks; ++r) {
            if (!(pending & (1u << r))) continue;
            const uint64_t w = ld_word(rx + r * p.slot_words);
            if (static_cast<uint32_t>(w >> 32) == e) {
                val[r] = __uint_as_float(static_cast<uint32_t>(w));
                pending &= ~(1u << r);
            }
        }
        if (pending && (spins & 63) == 63 && globaltimer_ns() - t0 > kPeerTimeoutNs) {
            atomicOr(status, kStatusPeerTimeout);
            return;
        }
    }
    float s = val[0];
    for (int r = 1; r < p.nranks; ++r) s = __fadd_rn(s, val[r]);
    v[i] = s;
}

// All-gather of `bytes` bytes per rank; with `pick`, the (index, value) pairs
// are reduced to the winner instead (value desc, index asc).
__global__ void __launch_bounds__(32) allgather_kernel(const __grid_constant__ CommParams p, const uint8_t *in,
                                                       uint8_t *out, int bytes, int pick) {
    pdl_launch_dependents();
    pdl_wait_prior_grid();
    __shared__ uint64_t s_e;
    __shared__ int s_timeout;
    const int t = threadIdx.x;
    uint8_t *own = p.win[p.rank];
    unsigned *status = reinterpret_cast<unsigned *>(own + p.off_status);
    if (t == 0) {
        uint64_t *ctr = reinterpret_cast<uint64_t *>(own + p.off_counters) + p.gmax;
        const uint64_t e = *ctr + 1;
        *ctr = e;
        s_e = e;
        s_timeout = 0;
    }
    __syncthreads();
    const uint64_t e = s_e;
    const uint64_t slot_off = p.off_ag + (e & 1) * kAgSlotBytes * kMaxRanks;
    uint32_t *mine = reinterpret_cast<uint32_t *>(own + slot_off + p.rank * kAgSlotBytes);
    const uint32_t *src = reinterpret_cast<const uint32_t *>(in);
    for (int i = t; i < bytes / 4; i += 32) mine[i] = src[i];
    __threadfence_system();
    __syncwarp();
    if (t < p.nranks && t != p.rank) {
        // every peer reads this rank's bytes from this rank's window
        uint64_t *peer_flags = reinterpret_cast<uint64_t *>(p.win[t] + p.off_agflags);
        st_release_sys(peer_flags + p.rank, e);
        const uint64_t *my_flags = reinterpret_cast<const uint64_t *>(own + p.off_agflags);
        if (!wait_flag(my_flags + t, e, status)) s_timeout = 1;
    }
    __syncthreads();
    if (s_timeout) return;
    if (!pick) {
        for (int r = 0; r < p.nranks; ++r) {
            const uint32_t *rs = reinterpret_cast<const uint32_t *>(p.win[r] + slot_off + r * kAgSlotBytes);
            uint32_t *dst = reinterpret_cast<uint32_t *>(out + r * bytes);
            for (int i = t; i < bytes / 4; i += 32) dst[i] = r == p.rank ? mine[i] : __ldcv(rs + i);
        }
        return;
    }
    if (t == 0) {
        int bi = 0;
        float bv = 0.0f;
        for (int r = 0; r < p.nranks; ++r) {
            const uint32_t *rs = reinterpret_cast<const uint32_t *>(p.win[r] + slot_off + r * kAgSlotBytes);
            const int ci = static_cast<int>(r == p.rank ? mine[0] : __ldcv(rs));
            const float cv = __uint_as_float(r == p.rank ? mine[1] : __ldcv(rs + 1));
            // sample_token's order (tp_llama.cpp:924): value desc, then index asc
            if (r == 0 || cv > bv || (cv == bv && ci < bi)) {
                bi = ci;
                bv = cv;
            }
        }
        reinterpret_cast<int *>(out)[0] = bi;
        reinterpret_cast<float *>(out)[1] = bv;
    }
}

}  // namespace

}  // namespace b200

using namespace b200;

struct b200_comm {
    int rank, nranks, device;
    int max_floats;
    uint8_t *win;               // own window
    size_t win_bytes;
    CommParams params;
    bool imported;
    uint8_t *mapped[kMaxRanks];  // IPC mappings to close
};

namespace {

int comm_fail(int code, const char *msg) { return report_error(code, msg); }

int set_device(int dev) {
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess) return comm_fail(kErrNoDev, "no CUDA device");
    if (cur != dev && cudaSetDevice(dev) != cudaSuccess) return comm_fail(kErrCuda, "cudaSetDevice failed");
    return 0;
}

uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

}  // namespace

extern "C" int b200_comm_handle_bytes(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

extern "C" int b200_comm_create(b200_comm_t **out, int rank, int nranks, int device, int max_floats) {
    if (!out) return comm_fail(kErrInval, "comm: null output");
    *out = nullptr;
    if (nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks)
        return comm_fail(kErrInval, "comm: need 0 <= rank < nranks <= 8");
    if (max_floats <= 0 || max_floats > (1 << 24)) return comm_fail(kErrInval, "comm: max_floats out of range");
    if (int rc = set_device(device)) return rc;
    b200_comm_t *c = static_cast<b200_comm_t *>(calloc(1, sizeof(b200_comm_t)));
    if (!c) return comm_fail(kErrNoMem, "comm: out of host memory");
    c->rank = rank;
    c->nranks = nranks;
    c->device = device;
    c->max_floats = max_floats;
    CommParams &p = c->params;
    p.rank = rank;
    p.nranks = nranks;
    p.gmax = (max_floats + kChunk - 1) / kChunk;
    p.slot_words = static_cast<uint64_t>(p.gmax) * kChunk;
    p.off_ag = align_up(2ull * kMaxRanks * p.slot_words * 8, 256);
    p.off_agflags = align_up(p.off_ag + 2ull * kAgSlotBytes * kMaxRanks, 256);
    p.off_counters = align_up(p.off_agflags + 8ull * kMaxRanks, 256);
    p.off_status = align_up(p.off_counters + 8ull * (p.gmax + 1), 256);
    c->win_bytes = align_up(p.off_status + 4, 4096);
    cudaError_t err = cudaMalloc(reinterpret_cast<void **>(&c->win), c->win_bytes);
    if (err == cudaSuccess) err = cudaMemset(c->win, 0, c->win_bytes);
    if (err == cudaSuccess) err = cudaDeviceSynchronize();
    if (err != cudaSuccess) {
        if (c->win) cudaFree(c->win);
        free(c);
        return comm_fail(kErrCuda, "comm: window allocation failed");
    }
    for (int r = 0; r < kMaxRanks; ++r) p.win[r] = nullptr;
    p.win[rank] = c->win;
    *out = c;
    return 0;
}

extern "C" int b200_comm_export(b200_comm_t *c, void *handle) {
    if (!c || !handle) return comm_fail(kErrInval, "comm: bad arguments");
    if (int rc = set_device(c->device)) return rc;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, c->win) != cudaSuccess) return comm_fail(kErrCuda, "comm: cudaIpcGetMemHandle failed");
    memcpy(handle, &h, sizeof h);
    return 0;
}

extern "C" int b200_comm_import(b200_comm_t *c, const void *handles) {
    if (!c || !handles) return comm_fail(kErrInval, "comm: bad arguments");
    if (c->imported) return comm_fail(kErrInval, "comm: handles already imported");
    if (int rc = set_device(c->device)) return rc;
    const uint8_t *hs = static_cast<const uint8_t *>(handles);
    for (int r = 0; r < c->nranks; ++r) {
        if (r == c->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, hs + static_cast<size_t>(r) * sizeof h, sizeof h);
        void *ptr = nullptr;
        const cudaError_t err = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (err != cudaSuccess) {
            char msg[160];
            snprintf(msg, sizeof msg, "comm: cannot map rank %d's window: %s", r, cudaGetErrorString(err));
            for (int q = 0; q < r; ++q)
                if (c->mapped[q]) cudaIpcCloseMemHandle(c->mapped[q]);
            return comm_fail(kErrCuda, msg);
        }
        c->mapped[r] = static_cast<uint8_t *>(ptr);
        c->params.win[r] = static_cast<uint8_t *>(ptr);
    }
    c->imported = true;
    return 0;
}

namespace {

int comm_launch_check(b200_comm_t *c) {
    if (!c) return comm_fail(kErrInval, "comm: not created");
    if (c->nranks > 1 && !c->imported) return comm_fail(kErrInval, "comm: peers' handles not imported");
    return set_device(c->device);
}

cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, cudaStream_t stream, cudaLaunchAttribute *attr) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = stream;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

}  // namespace

extern "C" int b200_allreduce_sum(b200_comm_t *c, uint64_t v, int len, void *stream) {
    if (int rc = comm_launch_check(c)) return rc;
    if (!v || v % 4 || len <= 0 || len > c->max_floats) return comm_fail(kErrInval, "allreduce: bad buffer or length");
    if (c->nranks == 1) return 0;  // comm_t short-circuits a single rank the same way (tp_llama.cpp:505)
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_config(dim3((len + kChunk - 1) / kChunk), dim3(kCommThreads),
                                        static_cast<cudaStream_t>(stream), attr);
    if (cudaLaunchKernelEx(&cfg, allreduce_kernel, c->params, reinterpret_cast<float *>(v), len) != cudaSuccess)
        return comm_fail(kErrCuda, "allreduce: launch failed");
    return 0;
}

namespace {

int gather(b200_comm_t *c, uint64_t in, uint64_t out, int bytes, void *stream, int pick) {
    if (int rc = comm_launch_check(c)) return rc;
    if (!in || !out || in % 4 || out % 4 || bytes <= 0 || bytes > kAgSlotBytes || bytes % 4)
        return comm_fail(kErrInval, "allgather: bad buffers or size");
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_config(dim3(1), dim3(32), static_cast<cudaStream_t>(stream), attr);
    if (c->nranks == 1) {
        // one rank: the gather is a copy, the pick is the rank's own pick
        const cudaError_t err = cudaMemcpyAsync(reinterpret_cast<void *>(out), reinterpret_cast<const void *>(in),
                                                static_cast<size_t>(bytes), cudaMemcpyDeviceToDevice,
                                                static_cast<cudaStream_t>(stream));
        return err == cudaSuccess ? 0 : comm_fail(kErrCuda, "allgather: copy failed");
    }
    if (cudaLaunchKernelEx(&cfg, allgather_kernel, c->params, reinterpret_cast<const uint8_t *>(in),
                           reinterpret_cast<uint8_t *>(out), bytes, pick) != cudaSuccess)
        return comm_fail(kErrCuda, "allgather: launch failed");
    return 0;
}

}  // namespace

extern "C" int b200_allgather(b200_comm_t *c, uint64_t in, uint64_t out, int bytes, void *stream) {
    return gather(c, in, out, bytes, stream, 0);
}

extern "C" int b200_allgather_pick(b200_comm_t *c, uint64_t in, uint64_t out, void *stream) {
    return gather(c, in, out, 8, stream, 1);
}

extern "C" int b200_comm_status(b200_comm_t *c, unsigned *status) {
    if (!c || !status) return comm_fail(kErrInval, "comm: bad arguments");
    if (int rc = set_device(c->device)) return rc;
    unsigned *dev = reinterpret_cast<unsigned *>(c->win + c->params.off_status);
    if (cudaMemcpy(status, dev, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return comm_fail(kErrCuda, "comm: status read failed");
    if (cudaMemset(dev, 0, 4) != cudaSuccess) return comm_fail(kErrCuda, "comm: status clear failed");
    return 0;
}

extern "C" int b200_comm_destroy(b200_comm_t *c) {
    if (!c) return 0;
    set_device(c->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < kMaxRanks; ++r)
        if (c->mapped[r]) cudaIpcCloseMemHandle(c->mapped[r]);
    if (c->win) cudaFree(c->win);
    free(c);
    return 0;
}

namespace b200 {

int comm_word_area(b200_comm_t *c, uint64_t *win_words[kMaxDecodeRanks], uint64_t *slot_words, unsigned **status,
                   int *rank, int *nranks) {
    if (!c || (c->nranks > 1 && !c->imported)) return kErrInval;
    for (int r = 0; r < kMaxDecodeRanks; ++r)
        win_words[r] = r < c->nranks ? reinterpret_cast<uint64_t *>(c->params.win[r]) : nullptr;
    *slot_words = c->params.slot_words;
    *status = reinterpret_cast<unsigned *>(c->win + c->params.off_status);
    *rank = c->rank;
    *nranks = c->nranks;
    return 0;
}

}  // namespace b200
