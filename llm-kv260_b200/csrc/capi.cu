// The C ABI: gemv_dev.h, gemv2_dev.h and udmabuf.h (drop-in replacements for
// board/kv260gemv/) and b200_engine.h (the runtime's engine_t call). Host
// code only; the kernels live in q4gemv.cu.
#include <cuda_runtime.h>

#include <cerrno>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <mutex>
#include <sched.h>

#include "../../include/b200_engine.h"
#include "../../include/gemv2_dev.h"
#include "../../include/gemv_dev.h"
#include "../../include/udmabuf.h"
#include "q4gemv.h"

using namespace b200;

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    return fail(kErrCuda, "%s: %s", what, cudaGetErrorString(e));
}

uint64_t now_ns() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return static_cast<uint64_t>(ts.tv_sec) * 1000000000ull + static_cast<uint64_t>(ts.tv_nsec);
}

int use_device(int dev) {
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess) return fail(kErrNoDev, "no CUDA device");
    if (cur != dev) {
        cudaError_t e = cudaSetDevice(dev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    }
    return 0;
}

constexpr int kDefaultTimeoutMs = 10000;
constexpr uint64_t kStageTimeoutNs = 2000000000ull;

// Poll an event until it completes, fails, or timeout_ms passes.
int wait_event(cudaEvent_t ev, int timeout_ms, uint64_t *elapsed_ns) {
    const uint64_t t0 = now_ns();
    const uint64_t limit = static_cast<uint64_t>(timeout_ms > 0 ? timeout_ms : kDefaultTimeoutMs) * 1000000ull;
    for (unsigned spins = 0;; ++spins) {
        const cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) return cuda_fail(e, "device work failed");
        if (now_ns() - t0 > limit) return fail(kErrTimeout, "wait timed out after %d ms", timeout_ms > 0 ? timeout_ms : kDefaultTimeoutMs);
        if (spins > 4096) sched_yield();
    }
    if (elapsed_ns) *elapsed_ns = now_ns() - t0;
    return 0;
}

// A kernel can only have given up on a stage if the call ran for at least
// the stage timeout; only then is the status word worth a device read.
int check_status_if_slow(uint64_t started_ns) {
    if (now_ns() - started_ns < kStageTimeoutNs) return 0;
    unsigned st = 0;
    if (read_status(&st) != 0) return fail(kErrCuda, "reading the device status failed");
    if (st) {
        clear_status();
        return fail(kErrTimeout, "a weight stage never arrived (status 0x%x); the output is incomplete", st);
    }
    return 0;
}

int parse_engine_name(const char *name, int *device) {
    static const char *known[] = {"gemv_q4_0", "gemv_fetch", "gemv_mac"};
    const char *colon = strchr(name, ':');
    const size_t len = colon ? static_cast<size_t>(colon - name) : strlen(name);
    bool ok = false;
    for (const char *k : known)
        if (strlen(k) == len && strncmp(k, name, len) == 0) ok = true;
    if (!ok) return -1;
    if (colon) {
        char *end = nullptr;
        const long v = strtol(colon + 1, &end, 10);
        if (!end || *end || v < 0) return -1;
        *device = static_cast<int>(v);
    } else if (cudaGetDevice(device) != cudaSuccess) {
        return -1;
    }
    return 0;
}

int launch_and_record(gemv_dev_t *d, const GemvLaunch &L) {
    if (int rc = use_device(d->fd)) return rc;
    const char *why = nullptr;
    if (gemv_validate(L, &why)) return fail(kErrInval, "gemv: %s", why);
    static const Tuning tuning;
    if (int rc = gemv_launch(L, tuning, static_cast<cudaStream_t>(d->stream)))
        return fail(rc, "gemv launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(d->done), static_cast<cudaStream_t>(d->stream));
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
    d->pending = 1;
    d->started_ns = now_ns();
    return 0;
}

}  // namespace

namespace b200 {
// Lets the other translation units of this library leave a message for
// b200_last_error() / gemv_dev_last_error().
int report_error(int code, const char *msg) { return fail(code, "%s", msg); }
}  // namespace b200

// =================================================================== gemv_dev.h

extern "C" int gemv_dev_open_named(gemv_dev_t *d, const char *name, int quiet) {
    if (!d || !name) return -1;
    memset(d, 0, sizeof *d);
    d->fd = -1;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
        if (!quiet) fprintf(stderr, "gemv_dev: no CUDA device for %s\n", name);
        fail(kErrNoDev, "no CUDA device");
        return -1;
    }
    int dev = 0;
    if (parse_engine_name(name, &dev) || dev >= count) {
        if (!quiet) fprintf(stderr, "gemv_dev: no engine named %s\n", name);
        fail(kErrNoDev, "no engine named %s", name);
        return -1;
    }
    if (use_device(dev)) {
        if (!quiet) fprintf(stderr, "gemv_dev: %s\n", g_err);
        return -1;
    }
    cudaStream_t s = nullptr;
    cudaEvent_t ev = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
        if (s) cudaStreamDestroy(s);
        if (!quiet) fprintf(stderr, "gemv_dev: cannot create a stream on device %d\n", dev);
        fail(kErrCuda, "stream/event creation failed");
        return -1;
    }
    d->fd = dev;
    d->stream = s;
    d->done = ev;
    d->owns_stream = 1;
    d->timeout_ms = kDefaultTimeoutMs;
    return 0;
}

extern "C" int gemv_dev_open(gemv_dev_t *d) { return gemv_dev_open_named(d, "gemv_q4_0", 0); }

extern "C" int gemv_dev_close(gemv_dev_t *d) {
    if (!d) return fail(kErrInval, "null engine");
    if (d->fd >= 0) {
        use_device(d->fd);
        if (d->done) {
            cudaEventSynchronize(static_cast<cudaEvent_t>(d->done));
            cudaEventDestroy(static_cast<cudaEvent_t>(d->done));
        }
        if (d->owns_stream && d->stream) cudaStreamDestroy(static_cast<cudaStream_t>(d->stream));
    }
    memset(d, 0, sizeof *d);
    d->fd = -1;
    return 0;
}

extern "C" int gemv_dev_start(gemv_dev_t *d, uint64_t w, uint64_t x, uint64_t y, int k, int rows) {
    if (!d || d->fd < 0) return fail(kErrInval, "engine not open");
    GemvLaunch L;
    L.region[0] = reinterpret_cast<const uint8_t *>(w);
    L.nregions = 1;
    L.rows = rows;
    L.k = k;
    L.layout = kLayoutRows;
    L.xmode = kXPacked;
    L.x = reinterpret_cast<const void *>(x);
    L.y = reinterpret_cast<float *>(y);
    return launch_and_record(d, L);
}

extern "C" int gemv_dev_start4(gemv_dev_t *d, const uint64_t w[4], uint64_t x, uint64_t y, int k, int rows) {
    if (!d || d->fd < 0) return fail(kErrInval, "engine not open");
    if (!w) return fail(kErrInval, "null region array");
    if (rows % 4) return fail(kErrInval, "gemv_dev_start4: rows %% 4 != 0");
    GemvLaunch L;
    for (int r = 0; r < 4; ++r) L.region[r] = reinterpret_cast<const uint8_t *>(w[r]);
    L.nregions = 4;
    L.rows = rows;
    L.k = k;
    L.layout = kLayoutRows;
    L.xmode = kXPacked;
    L.x = reinterpret_cast<const void *>(x);
    L.y = reinterpret_cast<float *>(y);
    return launch_and_record(d, L);
}

extern "C" int gemv_dev_wait(gemv_dev_t *d) {
    if (!d || d->fd < 0) return fail(kErrInval, "engine not open");
    if (!d->pending) return 0;
    if (int rc = use_device(d->fd)) return rc;
    if (int rc = wait_event(static_cast<cudaEvent_t>(d->done), d->timeout_ms, nullptr)) return rc;
    d->pending = 0;
    return check_status_if_slow(d->started_ns);
}

extern "C" int gemv_dev_run(gemv_dev_t *d, uint64_t w, uint64_t x, uint64_t y, int k, int rows) {
    if (int rc = gemv_dev_start(d, w, x, y, k, rows)) return rc;
    return gemv_dev_wait(d);
}

extern "C" int gemv_dev_set_stream(gemv_dev_t *d, void *stream) {
    if (!d || d->fd < 0) return fail(kErrInval, "engine not open");
    if (int rc = use_device(d->fd)) return rc;
    if (d->pending) {
        if (int rc = gemv_dev_wait(d)) return rc;
    }
    if (d->owns_stream && d->stream) cudaStreamDestroy(static_cast<cudaStream_t>(d->stream));
    d->stream = stream;  // NULL is the legacy default stream
    d->owns_stream = 0;
    return 0;
}

extern "C" int gemv_dev_status(gemv_dev_t *d, unsigned *status) {
    if (!d || d->fd < 0 || !status) return fail(kErrInval, "engine not open");
    if (int rc = use_device(d->fd)) return rc;
    if (read_status(status)) return fail(kErrCuda, "status read failed");
    return clear_status() ? fail(kErrCuda, "status clear failed") : 0;
}

extern "C" const char *gemv_dev_last_error(void) { return g_err; }

// ================================================================== gemv2_dev.h

extern "C" int gemv2_dev_open(gemv2_dev_t *d) {
    if (!d) return -1;
    memset(d, 0, sizeof *d);
    if (gemv_dev_open_named(&d->fetch, "gemv_fetch", 1)) return -1;
    if (gemv_dev_open_named(&d->mac, "gemv_mac", 0)) {
        gemv_dev_close(&d->fetch);
        return -1;
    }
    return 0;
}

extern "C" int gemv2_dev_close(gemv2_dev_t *d) {
    if (!d) return fail(kErrInval, "null engine");
    gemv_dev_close(&d->fetch);
    gemv_dev_close(&d->mac);
    d->fetched = 0;
    return 0;
}

extern "C" int gemv2_fetch_wait(gemv2_dev_t *d) {
    if (!d) return fail(kErrInval, "null engine");
    return gemv_dev_wait(&d->fetch);
}

extern "C" int gemv2_fetch_start(gemv2_dev_t *d, const uint64_t w[4], int k, int rows) {
    if (!d || d->fetch.fd < 0 || !w) return fail(kErrInval, "engine not open");
    if (int rc = gemv2_fetch_wait(d)) return rc;
    if (k <= 0 || k % 256 || k > kMaxK) return fail(kErrInval, "gemv2: k must be a multiple of 256 in [256, 8192]");
    if (rows <= 0 || rows % 8) return fail(kErrInval, "gemv2: rows %% 8 != 0");
    const uint8_t *regions[4];
    for (int r = 0; r < 4; ++r) {
        if (!w[r] || w[r] % 16) return fail(kErrInval, "gemv2: port regions must be 16-byte aligned");
        regions[r] = reinterpret_cast<const uint8_t *>(w[r]);
        d->w[r] = w[r];
    }
    d->k = k;
    d->rows = rows;
    d->fetched = 1;
    if (int rc = use_device(d->fetch.fd)) return rc;
    const size_t region_bytes = static_cast<size_t>(rows / 4) * (k / kQK) * kBlockBytes;
    if (prefetch_l2_launch(regions, 4, region_bytes, static_cast<cudaStream_t>(d->fetch.stream)))
        return fail(kErrCuda, "prefetch launch failed");
    cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(d->fetch.done), static_cast<cudaStream_t>(d->fetch.stream));
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
    d->fetch.pending = 1;
    d->fetch.started_ns = now_ns();
    return 0;
}

extern "C" int gemv2_mac_start(gemv2_dev_t *d, uint64_t x, uint64_t y, int k, int rows) {
    if (!d || d->mac.fd < 0) return fail(kErrInval, "engine not open");
    if (!d->fetched || d->k != k || d->rows != rows)
        return fail(kErrInval, "gemv2_mac_start: no pending fetch of a %dx%d matrix", rows, k);
    GemvLaunch L;
    for (int r = 0; r < 4; ++r) L.region[r] = reinterpret_cast<const uint8_t *>(d->w[r]);
    L.nregions = 4;
    L.rows = rows;
    L.k = k;
    L.layout = kLayoutPairs;
    L.xmode = kXPacked;
    L.x = reinterpret_cast<const void *>(x);
    L.y = reinterpret_cast<float *>(y);
    const int rc = launch_and_record(&d->mac, L);
    if (rc == 0) d->fetched = 0;
    return rc;
}

extern "C" int gemv2_mac_wait(gemv2_dev_t *d) {
    if (!d) return fail(kErrInval, "null engine");
    return gemv_dev_wait(&d->mac);
}

extern "C" int gemv2_mac_idle(gemv2_dev_t *d) {
    if (!d || d->mac.fd < 0) return fail(kErrInval, "engine not open");
    if (!d->mac.pending) return 1;
    if (int rc = use_device(d->mac.fd)) return rc;
    const cudaError_t e = cudaEventQuery(static_cast<cudaEvent_t>(d->mac.done));
    if (e == cudaSuccess) return 1;
    if (e == cudaErrorNotReady) return 0;
    return cuda_fail(e, "device work failed");
}

extern "C" int gemv2_drain(gemv2_dev_t *d) {
    if (!d) return fail(kErrInval, "null engine");
    d->fetched = 0;
    if (int rc = gemv_dev_wait(&d->fetch)) return rc;
    return gemv_dev_wait(&d->mac);
}

// ==================================================================== udmabuf.h

namespace {

struct Pool {
    uint8_t *host;
    uint8_t *dev;
    size_t size;
    int device;
};

std::mutex g_pool_mu;
Pool g_pools[32];
int g_npools = 0;

int find_pool(const void *p, size_t len, Pool *out) {
    std::lock_guard<std::mutex> lk(g_pool_mu);
    const uint8_t *q = static_cast<const uint8_t *>(p);
    for (int i = 0; i < g_npools; ++i) {
        const Pool &pl = g_pools[i];
        if (q >= pl.host && q + len <= pl.host + pl.size) {
            *out = pl;
            return 0;
        }
    }
    return fail(kErrInval, "udmabuf: %p..+%zu is not inside an open pool", p, len);
}

}  // namespace

extern "C" int udmabuf_open_size(udmabuf_t *b, const char *name, size_t size, int device) {
    if (!b || !name || size == 0) return fail(kErrInval, "udmabuf_open: bad arguments");
    memset(b, 0, sizeof *b);
    b->fd = -1;
    if (use_device(device)) {
        fprintf(stderr, "udmabuf: %s: %s\n", name, g_err);
        return -1;
    }
    void *dev = nullptr, *host = nullptr;
    cudaError_t e = cudaMalloc(&dev, size);
    if (e == cudaSuccess) e = cudaHostAlloc(&host, size, cudaHostAllocDefault);
    if (e != cudaSuccess) {
        if (dev) cudaFree(dev);
        fprintf(stderr, "udmabuf: %s: cannot allocate %zu bytes: %s\n", name, size, cudaGetErrorString(e));
        cuda_fail(e, "udmabuf allocation");
        return -1;
    }
    memset(host, 0, size);
    cudaMemset(dev, 0, size);
    {
        std::lock_guard<std::mutex> lk(g_pool_mu);
        if (g_npools == 32) {
            cudaFree(dev);
            cudaFreeHost(host);
            fail(kErrNoMem, "udmabuf: too many open pools");
            return -1;
        }
        g_pools[g_npools++] = Pool{static_cast<uint8_t *>(host), static_cast<uint8_t *>(dev), size, device};
    }
    b->fd = device;
    b->base = static_cast<uint8_t *>(host);
    b->phys = reinterpret_cast<uint64_t>(dev);
    b->size = size;
    b->used = 0;
    return 0;
}

extern "C" int udmabuf_open(udmabuf_t *b, const char *name) {
    if (!b || !name) return fail(kErrInval, "udmabuf_open: bad arguments");
    char var[96];
    snprintf(var, sizeof var, "UDMABUF_SIZE_%s", name);
    for (char *c = var; *c; ++c)
        if (*c >= 'a' && *c <= 'z') *c = static_cast<char>(*c - 'a' + 'A');
    size_t size = static_cast<size_t>(256) << 20;
    if (const char *v = getenv(var)) {
        const unsigned long long s = strtoull(v, nullptr, 0);
        if (s) size = static_cast<size_t>(s);
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        fprintf(stderr, "udmabuf: no CUDA device for %s\n", name);
        return -1;
    }
    return udmabuf_open_size(b, name, size, dev);
}

extern "C" int udmabuf_close(udmabuf_t *b) {
    if (!b) return fail(kErrInval, "null pool");
    if (b->base) {
        std::lock_guard<std::mutex> lk(g_pool_mu);
        for (int i = 0; i < g_npools; ++i) {
            if (g_pools[i].host == b->base) {
                use_device(g_pools[i].device);
                cudaFree(g_pools[i].dev);
                cudaFreeHost(g_pools[i].host);
                g_pools[i] = g_pools[--g_npools];
                break;
            }
        }
    }
    memset(b, 0, sizeof *b);
    b->fd = -1;
    return 0;
}

extern "C" void *udmabuf_alloc(udmabuf_t *b, size_t size, size_t align) {
    if (!b || !b->base || align == 0 || (align & (align - 1))) return nullptr;
    const size_t start = (b->used + align - 1) & ~(align - 1);
    if (start + size > b->size) return nullptr;
    b->used = start + size;
    return b->base + start;
}

extern "C" int udmabuf_clean(const void *p, size_t len) {
    Pool pl;
    if (int rc = find_pool(p, len, &pl)) return rc;
    const size_t off = static_cast<size_t>(static_cast<const uint8_t *>(p) - pl.host);
    const cudaError_t e = cudaMemcpy(pl.dev + off, p, len, cudaMemcpyHostToDevice);
    return e == cudaSuccess ? 0 : cuda_fail(e, "udmabuf_clean");
}

extern "C" int udmabuf_invalidate(const void *p, size_t len) {
    Pool pl;
    if (int rc = find_pool(p, len, &pl)) return rc;
    const size_t off = static_cast<size_t>(static_cast<const uint8_t *>(p) - pl.host);
    const cudaError_t e = cudaMemcpy(const_cast<void *>(p), pl.dev + off, len, cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? 0 : cuda_fail(e, "udmabuf_invalidate");
}

// =============================================================== b200_engine.h

struct b200_engine {
    int device;
    cudaStream_t own;
    cudaStream_t stream;
    cudaStream_t side;
    cudaEvent_t fork;
    cudaEvent_t done;
    uint8_t *xscratch;  // quantised x for the two-kernel f32 path
    void *sel_scratch;  // argmax candidates
    void *fsel_scratch; // fused greedy pick: per-CTA candidates + ticket
    b200_engine_config_t cfg;
};

namespace {

constexpr size_t kXScratchBytes = kMaxK + 4 * (kMaxK / kQK);

Tuning tuning_of(const b200_engine_config_t &c) {
    Tuning t;
    t.stage_bytes = c.stage_bytes;
    t.stages = c.stages;
    t.ctas_per_sm = c.ctas_per_sm;
    t.xreg_chunks = c.xreg_chunks;
    t.kslices = c.kslices;
    return t;
}

// One engine GEMV: validate, then launch the kernel of W's layout.
int engine_gemv(b200_engine_t *e, const b200_qmat_t *W, int xmode, const void *x, uint64_t y, int *sel_out = nullptr,
                int sel_base = 0) {
    if (!e) return fail(kErrInval, "engine not open");
    if (!W) return fail(kErrInval, "null matrix");
    const char *why = nullptr;
    if (W->layout == B200_LAYOUT_TILES) {
        TileLaunch L;
        L.w = reinterpret_cast<const uint8_t *>(W->w);
        L.rows = W->rows;
        L.k = W->k;
        L.xmode = xmode;
        L.x = x;
        L.y = reinterpret_cast<float *>(y);
        L.round_mode = e->cfg.round_mode;
        L.l2_policy = e->cfg.l2_policy;
        L.pdl = e->cfg.pdl != 0;
        L.sel_out = sel_out;
        L.sel_base = sel_base;
        L.sel_scratch = e->fsel_scratch;
        if (tile_validate(L, &why)) return fail(kErrInval, "gemv %dx%d: %s", W->rows, W->k, why);
        if (int rc = use_device(e->device)) return rc;
        if (tile_launch(L, tuning_of(e->cfg), e->stream))
            return fail(kErrCuda, "gemv launch failed: %s", cudaGetErrorString(cudaGetLastError()));
        return 0;
    }
    if (W->layout != B200_LAYOUT_ROWS) return fail(kErrInval, "unknown matrix layout %d", W->layout);
    if (sel_out) return fail(kErrInval, "the fused greedy pick needs a tile-layout matrix");
    GemvLaunch L;
    L.region[0] = reinterpret_cast<const uint8_t *>(W->w);
    L.nregions = 1;
    L.rows = W->rows;
    L.k = W->k;
    L.layout = kLayoutRows;
    L.xmode = xmode;
    L.x = x;
    L.y = reinterpret_cast<float *>(y);
    L.round_mode = e->cfg.round_mode;
    L.l2_policy = e->cfg.l2_policy;
    L.pdl = e->cfg.pdl != 0;
    if (gemv_validate(L, &why)) return fail(kErrInval, "gemv %dx%d: %s", W->rows, W->k, why);
    if (int rc = use_device(e->device)) return rc;
    if (gemv_launch(L, tuning_of(e->cfg), e->stream))
        return fail(kErrCuda, "gemv launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    return 0;
}

// Shape checks shared by the f32 path (before it quantises into scratch).
int check_qmat(const b200_qmat_t *W) {
    if (!W) return fail(kErrInval, "null matrix");
    if (W->k <= 0 || W->k % 256 || W->k > kMaxK) return fail(kErrInval, "gemv %dx%d: k must be a multiple of 256 in [256, 8192]", W->rows, W->k);
    if (W->rows <= 0) return fail(kErrInval, "gemv: rows must be positive");
    return 0;
}

int prefetch_on_side(b200_engine_t *e, const b200_qmat_t *W) {
    if (W->rows <= 0 || W->k <= 0 || W->k % kQK || W->w % 16) return fail(kErrInval, "prefetch: bad matrix");
    cudaError_t err = cudaEventRecord(e->fork, e->stream);
    if (err == cudaSuccess) err = cudaStreamWaitEvent(e->side, e->fork, 0);
    if (err != cudaSuccess) return cuda_fail(err, "prefetch fork");
    const uint8_t *r[1] = {reinterpret_cast<const uint8_t *>(W->w)};
    const size_t bytes = W->layout == B200_LAYOUT_TILES ? tiled_bytes(W->rows, W->k)
                                                        : static_cast<size_t>(W->rows) * (W->k / kQK) * kBlockBytes;
    return prefetch_l2_launch(r, 1, bytes, e->side) ? fail(kErrCuda, "prefetch launch failed") : 0;
}

}  // namespace

extern "C" int b200_device_count(void) {
    int n = 0;
    return cudaGetDeviceCount(&n) == cudaSuccess ? n : 0;
}

extern "C" const char *b200_last_error(void) { return g_err; }

extern "C" int b200_engine_open(b200_engine_t **out, int device) {
    if (!out) return fail(kErrInval, "null output");
    *out = nullptr;
    const int n = b200_device_count();
    if (n == 0) return fail(kErrNoDev, "no CUDA device");
    if (device < 0 || device >= n) return fail(kErrNoDev, "device %d out of range (%d devices)", device, n);
    if (int rc = use_device(device)) return rc;
    b200_engine_t *e = static_cast<b200_engine_t *>(calloc(1, sizeof(b200_engine_t)));
    if (!e) return fail(kErrNoMem, "out of host memory");
    e->device = device;
    cudaError_t err = cudaStreamCreateWithFlags(&e->own, cudaStreamNonBlocking);
    if (err == cudaSuccess) err = cudaStreamCreateWithFlags(&e->side, cudaStreamNonBlocking);
    if (err == cudaSuccess) err = cudaEventCreateWithFlags(&e->fork, cudaEventDisableTiming);
    if (err == cudaSuccess) err = cudaEventCreateWithFlags(&e->done, cudaEventDisableTiming);
    if (err == cudaSuccess) err = cudaMalloc(reinterpret_cast<void **>(&e->xscratch), kXScratchBytes);
    if (err == cudaSuccess) err = cudaMalloc(&e->sel_scratch, static_cast<size_t>(argmax_scratch_bytes()));
    if (err == cudaSuccess) err = cudaMalloc(&e->fsel_scratch, static_cast<size_t>(tile_select_scratch_bytes()));
    if (err == cudaSuccess) err = cudaMemset(e->fsel_scratch, 0, static_cast<size_t>(tile_select_scratch_bytes()));
    if (err != cudaSuccess) {
        b200_engine_close(e);
        return cuda_fail(err, "engine set-up");
    }
    e->stream = e->own;
    e->cfg.stage_bytes = 16384;
    e->cfg.stages = 4;
    e->cfg.ctas_per_sm = 2;
    e->cfg.l2_policy = kL2EvictFirst;
    e->cfg.pdl = 1;
    e->cfg.round_mode = kRoundContract;
    e->cfg.fuse_quantize = 0;
    e->cfg.prefetch_next = 0;
    e->cfg.xreg_chunks = 8;
    e->cfg.kslices = 1;
    *out = e;
    return 0;
}

extern "C" int b200_engine_close(b200_engine_t *e) {
    if (!e) return 0;
    use_device(e->device);
    if (e->stream) cudaStreamSynchronize(e->stream);
    if (e->side) cudaStreamSynchronize(e->side);
    if (e->xscratch) cudaFree(e->xscratch);
    if (e->sel_scratch) cudaFree(e->sel_scratch);
    if (e->fsel_scratch) cudaFree(e->fsel_scratch);
    if (e->fork) cudaEventDestroy(e->fork);
    if (e->done) cudaEventDestroy(e->done);
    if (e->side) cudaStreamDestroy(e->side);
    if (e->own) cudaStreamDestroy(e->own);
    free(e);
    return 0;
}

extern "C" int b200_engine_get_config(b200_engine_t *e, b200_engine_config_t *cfg) {
    if (!e || !cfg) return fail(kErrInval, "bad arguments");
    *cfg = e->cfg;
    return 0;
}

extern "C" int b200_engine_set_config(b200_engine_t *e, const b200_engine_config_t *cfg) {
    if (!e || !cfg) return fail(kErrInval, "bad arguments");
    if (cfg->stage_bytes < 16 || cfg->stages < 1 || cfg->stages > 8 || cfg->ctas_per_sm < 1 || cfg->ctas_per_sm > 32)
        return fail(kErrInval, "config out of range");
    if (cfg->l2_policy < 0 || cfg->l2_policy > 2 || cfg->round_mode < 0 || cfg->round_mode > 1)
        return fail(kErrInval, "config out of range");
    if (cfg->kslices != 1 && cfg->kslices != 2 && cfg->kslices != 4) return fail(kErrInval, "kslices must be 1, 2 or 4");
    e->cfg = *cfg;
    return 0;
}

extern "C" int b200_engine_set_stream(b200_engine_t *e, void *stream) {
    if (!e) return fail(kErrInval, "engine not open");
    e->stream = static_cast<cudaStream_t>(stream);  // NULL is the legacy default stream
    return 0;
}

extern "C" void *b200_engine_stream(b200_engine_t *e) { return e ? static_cast<void *>(e->stream) : nullptr; }

extern "C" int b200_quantize_q8_0(b200_engine_t *e, uint64_t x, uint64_t xpacked, int k) {
    if (!e) return fail(kErrInval, "engine not open");
    if (int rc = use_device(e->device)) return rc;
    if (k <= 0 || k % kQK) return fail(kErrInval, "quantize: k must be a positive multiple of 32");
    if (x % 16 || xpacked % 16) return fail(kErrInval, "quantize: x and xpacked must be 16-byte aligned");
    if (quantize_launch(reinterpret_cast<const float *>(x), reinterpret_cast<uint8_t *>(xpacked), k, e->cfg.round_mode,
                        e->stream, e->cfg.pdl != 0))
        return fail(kErrCuda, "quantize launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    return 0;
}

extern "C" int b200_gemv_q8(b200_engine_t *e, const b200_qmat_t *W, uint64_t xpacked, uint64_t y,
                            const b200_qmat_t *next) {
    if (int rc = engine_gemv(e, W, kXPacked, reinterpret_cast<const void *>(xpacked), y)) return rc;
    if (next && e->cfg.prefetch_next) return prefetch_on_side(e, next);
    return 0;
}

extern "C" int b200_gemv_f32(b200_engine_t *e, const b200_qmat_t *W, uint64_t x, uint64_t y,
                             const b200_qmat_t *next) {
    if (!e) return fail(kErrInval, "engine not open");
    if (int rc = check_qmat(W)) return rc;
    if (!e->cfg.fuse_quantize) {
        // The scratch buffer holds k <= 8192, checked above.
        if (x % 16) return fail(kErrInval, "x must be 16-byte aligned");
        if (int rc = b200_quantize_q8_0(e, x, reinterpret_cast<uint64_t>(e->xscratch), W->k)) return rc;
        return b200_gemv_q8(e, W, reinterpret_cast<uint64_t>(e->xscratch), y, next);
    }
    if (int rc = engine_gemv(e, W, kXF32, reinterpret_cast<const void *>(x), y)) return rc;
    if (next && e->cfg.prefetch_next) return prefetch_on_side(e, next);
    return 0;
}

extern "C" int b200_gemv_argmax_f32(b200_engine_t *e, const b200_qmat_t *W, uint64_t x, uint64_t y, int index_base,
                                    uint64_t out) {
    if (!e) return fail(kErrInval, "engine not open");
    if (int rc = check_qmat(W)) return rc;
    if (!out || out % 8) return fail(kErrInval, "out must be 8-byte aligned");
    if (W->layout != B200_LAYOUT_TILES) return fail(kErrInval, "the fused greedy pick needs a tile-layout matrix");
    int *sel = reinterpret_cast<int *>(out);
    if (!e->cfg.fuse_quantize) {
        if (x % 16) return fail(kErrInval, "x must be 16-byte aligned");
        if (int rc = b200_quantize_q8_0(e, x, reinterpret_cast<uint64_t>(e->xscratch), W->k)) return rc;
        return engine_gemv(e, W, kXPacked, e->xscratch, y, sel, index_base);
    }
    return engine_gemv(e, W, kXF32, reinterpret_cast<const void *>(x), y, sel, index_base);
}

extern "C" uint64_t b200_tiled_bytes(int rows, int k) { return static_cast<uint64_t>(tiled_bytes(rows, k)); }

extern "C" int b200_repack_q4_0(b200_engine_t *e, uint64_t src, int rows, int k, uint64_t dst) {
    if (!e) return fail(kErrInval, "engine not open");
    if (tiled_bytes(rows, k) == 0) return fail(kErrInval, "repack %dx%d: k must be a multiple of 256", rows, k);
    if (src % 2 || dst % 16) return fail(kErrInval, "repack: src must be 2-byte and dst 16-byte aligned");
    if (int rc = use_device(e->device)) return rc;
    if (repack_launch(reinterpret_cast<const uint8_t *>(src), rows, k, reinterpret_cast<uint8_t *>(dst), e->stream))
        return fail(kErrCuda, "repack launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    return 0;
}

extern "C" int b200_argmax_f32(b200_engine_t *e, uint64_t y, int n, int index_base, uint64_t out) {
    if (!e) return fail(kErrInval, "engine not open");
    if (!y || n <= 0 || !out || y % 4 || out % 4) return fail(kErrInval, "argmax: bad arguments");
    if (int rc = use_device(e->device)) return rc;
    int *oi = reinterpret_cast<int *>(out);
    if (argmax_launch(reinterpret_cast<const float *>(y), n, index_base, e->sel_scratch, oi,
                      reinterpret_cast<float *>(oi + 1), e->stream, e->cfg.pdl != 0))
        return fail(kErrCuda, "argmax launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    return 0;
}

extern "C" int b200_prefetch(b200_engine_t *e, const b200_qmat_t *W) {
    if (!e || !W) return fail(kErrInval, "bad arguments");
    if (int rc = use_device(e->device)) return rc;
    return prefetch_on_side(e, W);
}

extern "C" int b200_engine_sync(b200_engine_t *e, int timeout_ms) {
    if (!e) return fail(kErrInval, "engine not open");
    if (int rc = use_device(e->device)) return rc;
    cudaError_t err = cudaEventRecord(e->done, e->stream);
    if (err != cudaSuccess) return cuda_fail(err, "cudaEventRecord");
    if (int rc = wait_event(e->done, timeout_ms, nullptr)) return rc;
    err = cudaEventRecord(e->done, e->side);
    if (err != cudaSuccess) return cuda_fail(err, "cudaEventRecord");
    return wait_event(e->done, timeout_ms, nullptr);
}

extern "C" int b200_engine_status(b200_engine_t *e, unsigned *status) {
    if (!e || !status) return fail(kErrInval, "bad arguments");
    if (int rc = use_device(e->device)) return rc;
    if (read_status(status)) return fail(kErrCuda, "status read failed");
    return clear_status() ? fail(kErrCuda, "status clear failed") : 0;
}

extern "C" int b200_gemv_plan(b200_engine_t *e, int rows, int k, int layout, int fused_f32, int *grid,
                              int *smem_bytes) {
    if (!e) return fail(kErrInval, "engine not open");
    if (int rc = use_device(e->device)) return rc;
    static const uint8_t aligned[16] __attribute__((aligned(16))) = {};
    float *ydummy = reinterpret_cast<float *>(const_cast<uint8_t *>(aligned));
    if (layout == B200_LAYOUT_TILES) {
        TileLaunch L;
        L.w = aligned;
        L.rows = rows;
        L.k = k;
        L.xmode = fused_f32 ? kXF32 : kXPacked;
        L.x = aligned;
        L.y = ydummy;
        if (int rc = tile_grid(L, tuning_of(e->cfg), grid, smem_bytes)) return fail(rc, "no plan for %dx%d", rows, k);
        return 0;
    }
    GemvLaunch L;
    L.region[0] = aligned;
    L.rows = rows;
    L.k = k;
    L.xmode = fused_f32 ? kXF32 : kXPacked;
    L.x = aligned;
    L.y = ydummy;
    if (int rc = gemv_grid(L, tuning_of(e->cfg), grid, smem_bytes)) return fail(rc, "no plan for %dx%d", rows, k);
    return 0;
}

// ----------------------------------------------------------------- graphs

struct b200_graph {
    int device;
    cudaGraph_t graph;
    cudaGraphExec_t exec;
};

extern "C" int b200_capture_begin(b200_engine_t *e) {
    if (!e) return fail(kErrInval, "engine not open");
    if (int rc = use_device(e->device)) return rc;
    if (e->stream == nullptr) return fail(kErrInval, "capture needs a stream of its own, not the legacy default");
    const cudaError_t err = cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal);
    return err == cudaSuccess ? 0 : cuda_fail(err, "cudaStreamBeginCapture");
}

extern "C" int b200_capture_end(b200_engine_t *e, b200_graph_t **g) {
    if (!e || !g) return fail(kErrInval, "bad arguments");
    *g = nullptr;
    if (int rc = use_device(e->device)) return rc;
    cudaGraph_t graph = nullptr;
    cudaError_t err = cudaStreamEndCapture(e->stream, &graph);
    if (err != cudaSuccess) return cuda_fail(err, "cudaStreamEndCapture");
    cudaGraphExec_t exec = nullptr;
    err = cudaGraphInstantiate(&exec, graph, 0);
    if (err != cudaSuccess) {
        cudaGraphDestroy(graph);
        return cuda_fail(err, "cudaGraphInstantiate");
    }
    b200_graph_t *out = static_cast<b200_graph_t *>(calloc(1, sizeof(b200_graph_t)));
    if (!out) {
        cudaGraphExecDestroy(exec);
        cudaGraphDestroy(graph);
        return fail(kErrNoMem, "out of host memory");
    }
    out->device = e->device;
    out->graph = graph;
    out->exec = exec;
    *g = out;
    return 0;
}

extern "C" int b200_graph_launch(b200_engine_t *e, b200_graph_t *g) {
    if (!e || !g) return fail(kErrInval, "bad arguments");
    if (g->device != e->device) return fail(kErrInval, "graph and engine are on different devices");
    if (int rc = use_device(e->device)) return rc;
    const cudaError_t err = cudaGraphLaunch(g->exec, e->stream);
    return err == cudaSuccess ? 0 : cuda_fail(err, "cudaGraphLaunch");
}

extern "C" int b200_graph_destroy(b200_graph_t *g) {
    if (!g) return 0;
    use_device(g->device);
    if (g->exec) cudaGraphExecDestroy(g->exec);
    if (g->graph) cudaGraphDestroy(g->graph);
    free(g);
    return 0;
}

extern "C" int b200_copy_async(b200_engine_t *e, uint64_t dst, uint64_t src, uint64_t bytes) {
    if (!e) return fail(kErrInval, "engine not open");
    if (int rc = use_device(e->device)) return rc;
    const cudaError_t err = cudaMemcpyAsync(reinterpret_cast<void *>(dst), reinterpret_cast<const void *>(src),
                                            static_cast<size_t>(bytes), cudaMemcpyDefault, e->stream);
    return err == cudaSuccess ? 0 : cuda_fail(err, "cudaMemcpyAsync");
}
