// Q4_0 x Q8_0 GEMV for sm_100a, bit-exact to the reference contract
// src/llm_kv260/q4_0.py (gemv_q4_0, lines 151-182).
//
// The contract's order fixes the parallel structure: block b of a row feeds
// lane b mod 8, each lane is a sequential float32 chain over its blocks, and
// the 8 lanes meet in one adjacent-pair tree. So a CTA of 8 warps maps
//     warp w      <->  lane w (block position w inside every 144-byte chunk)
//     thread i    <->  row i of a 32-row group
// and every thread runs one lane chain of one row on its own: no shuffles,
// no order bookkeeping. The tree is done once per row group through shared
// memory, in tree_sum's order.
//
// Data path:
//   * Weights stay in the GGUF layout (rows of 18-byte blocks; 8 blocks make a
//     16-byte-aligned 144-byte chunk). A tiled TMA tensor map views them as
//     [chunk][row][byte of chunk]; one cp.async.bulk.tensor per stage (issued
//     by one thread, no multicast) lands 32 rows x C chunks in shared memory
//     as [C][32][144], completing on an mbarrier of an S-deep ring. Rows past
//     the end come back zero-filled.
//   * In that layout the 32 rows of a chunk sit 144 bytes apart, so the 32
//     threads of a warp reading one block offset hit 8 distinct 16-byte bank
//     groups per quarter warp: every weight read is a conflict-free 128-bit
//     load. Block w of a chunk lies in the 16-byte words at 16w and 16w+16,
//     and because w is the warp index the extraction shifts are compile-time
//     constants (the body is instantiated per lane).
//   * x (Q8_0) is identical for all rows: staged once per CTA in shared
//     memory (quantised there from float32 when the caller passes float32),
//     then held in registers when K <= 2048 (8 blocks per lane), else read by
//     warp-wide broadcast. The block dot is 8 __dp4a: sum(n * x) - 8 * sum(x).
//   * t = (f32(sumi) * f32(dw)) * f32(dx) as two rounded multiplies, then
//     lane = lane + t: __fmul_rn / __fadd_rn keep nvcc from fusing them.
#include <cuda.h>
#include <cuda_fp16.h>

#include <atomic>
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace b200 {

__device__ unsigned g_status;

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;  // one warp per lane: kWarps == kLanes
constexpr int kGroupRows = 32;         // rows per group: one per thread of a warp
constexpr int kChunkRowsBytes = kGroupRows * kChunkBytes;  // one chunk of a row group: 4608 B
constexpr int kMaxStages = 8;
constexpr int kBarBytes = 64;                           // kMaxStages mbarriers
constexpr int kRedBytes = 2 * kWarps * kGroupRows * 4;  // double-buffered lane sums
constexpr int kSmemAlign = 128;                         // TMA destination alignment

static_assert(kWarps == kLanes, "one warp per contract lane");

struct alignas(64) GemvParams {
    CUtensorMap tmap[4];    // one per region
    float *y;
    const void *x;
    int rows_per_region;
    int units_per_region;   // rows (ROWS) or row pairs (PAIRS)
    int k, nb, nch;         // nch = 144-byte chunks per row
    int groups_per_region;  // 32-row groups
    int ctas_per_region;
    int cps;                // chunks per stage
    int slices;             // stages per group = ceil(nch / cps)
    int slot_bytes;         // cps * 4608
    int stages;             // ring depth
    int xarea_bytes;        // shared bytes for x
    int round_mode;
    int l2_policy;
    unsigned *status;
};

// The contract's block term for the block at byte 18*L of the 144-byte chunk
// at `chunk` (shared memory): t = (f32(sumi) * f32(dw)) * f32(dx).
template <int L>
__device__ __forceinline__ float block_term(const uint8_t *chunk, const XBlock &xb) {
    const uint4 a = *reinterpret_cast<const uint4 *>(chunk + 16 * L);
    const uint4 c = *reinterpret_cast<const uint4 *>(chunk + 16 * L + 16);
    const uint32_t win[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
    // The block starts at byte 2L of the window: scale in bytes 2L..2L+1,
    // nibble word j in bytes 2L+2+4j..2L+5+4j.
    constexpr int kD = L / 2, kDShift = 16 * (L & 1);
    constexpr int kN = (L + 1) / 2, kNShift = 16 * ((L + 1) & 1);
    const uint32_t dbits = (win[kD] >> kDShift) & 0xffffu;
    uint32_t n[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        if constexpr (kNShift == 0) n[j] = win[kN + j];
        else n[j] = __funnelshift_r(win[kN + j], win[kN + j + 1], kNShift);
    }
    return block_term_words(n, dbits, xb);
}

// Stage s of this CTA (row group g0 + s / slices, K-slice s % slices): one
// tiled TMA load of 32 rows x cps chunks. Called by one thread.
template <int LAYOUT>
__device__ __forceinline__ void issue_stage(const GemvParams &p, uint64_t *bars, uint8_t *ring, int region, int g0,
                                            int s, uint64_t policy) {
    const int g = g0 + s / p.slices, c0 = (s % p.slices) * p.cps;
    const int slot = s % p.stages;
    mbar_arrive_expect_tx(&bars[slot], static_cast<uint32_t>(p.slot_bytes));
    if constexpr (LAYOUT == kLayoutPairs)
        tma_load_4d(ring + slot * p.slot_bytes, &p.tmap[region], 0, 0, g * (kGroupRows / 2), c0, &bars[slot], policy);
    else
        tma_load_3d(ring + slot * p.slot_bytes, &p.tmap[region], 0, g * kGroupRows, c0, &bars[slot], policy);
}

// Everything after set-up, for the warp that owns lane L. A stage is p.cps
// chunks of a 32-row group; x is read from shared memory by broadcast. The
// chunk loop is deliberately not unrolled: eight lane-specialised bodies have
// to fit the instruction cache together.
template <int LAYOUT, int L>
__device__ __forceinline__ void gemv_body(const GemvParams &p, uint64_t *bars, float *red, const uint8_t *xs,
                                          uint8_t *ring, int region, int g0, int g1, uint64_t policy,
                                          int *s_abort) {
    constexpr int M = LAYOUT == kLayoutPairs ? 2 : 1;  // rows per unit
    constexpr int UPG = kGroupRows / M;                // units per group
    const int lane = threadIdx.x & 31;
    const int S = p.stages;
    const int nst = (g1 - g0) * p.slices;

    float acc = 0.0f;
    int s = 0;
    for (; s < nst; ++s) {
        const int slot = s % S;
        const int gi = s / p.slices, sl = s % p.slices;
        if (!wait_stage(&bars[slot], static_cast<uint32_t>((s / S) & 1), p.status)) *s_abort = 1;
        const uint8_t *rowbase = ring + slot * p.slot_bytes + lane * kChunkBytes;
        const int c0 = sl * p.cps, cc = min(p.cps, p.nch - c0);
#pragma unroll 1
        for (int j = 0; j < cc; ++j) {
            XBlock xb;
            load_xblock_smem(xs, p.k, 8 * (c0 + j) + L, xb);
            acc = __fadd_rn(acc, block_term<L>(rowbase + j * kChunkRowsBytes, xb));
        }
        const bool last_slice = sl == p.slices - 1;
        float *rbuf = red + (gi & 1) * (kWarps * kGroupRows);
        if (last_slice) {
            rbuf[L * kGroupRows + lane] = acc;
            acc = 0.0f;
        }
        __syncthreads();
        if (*s_abort) break;
        if (L == 0 && lane == 0 && s + S < nst) issue_stage<LAYOUT>(p, bars, ring, region, g0, s + S, policy);
        if (L == 1 && last_slice) {
            // tree_sum over the 8 lanes (q4_0.py:67-78): ((0+1)+(2+3))+((4+5)+(6+7)).
            const float *r = rbuf + lane;
            const float yv = tree8(r[0 * kGroupRows], r[1 * kGroupRows], r[2 * kGroupRows], r[3 * kGroupRows],
                                   r[4 * kGroupRows], r[5 * kGroupRows], r[6 * kGroupRows], r[7 * kGroupRows]);
            // group row `lane` is unit lane / M, member lane % M; a pair is rows
            // u and u + units_per_region (gemv2_dev.h:46-49)
            const int u = (g0 + gi) * UPG + (M == 2 ? lane >> 1 : lane);
            if (u < p.units_per_region)
                p.y[region * p.rows_per_region + u + (M == 2 ? (lane & 1) * p.units_per_region : 0)] = yv;
        }
    }
    if (s < nst && L == 0 && lane == 0) {
        // Aborted on a stage timeout: let copies already in flight land (each
        // wait bounded) before the CTA's shared memory goes away.
        const int issued = min(nst, s + S);
        for (int r = s; r < issued; ++r) (void)wait_stage(&bars[r % S], static_cast<uint32_t>((r / S) & 1), p.status);
    }
}

template <int LAYOUT, int XMODE>
__global__ void __launch_bounds__(kThreads, 1) q4_gemv_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ int s_abort;
    uint8_t *ring = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + kSmemAlign - 1) & ~static_cast<uintptr_t>(kSmemAlign - 1));
    uint64_t *bars = reinterpret_cast<uint64_t *>(ring + p.stages * p.slot_bytes);
    float *red = reinterpret_cast<float *>(ring + p.stages * p.slot_bytes + kBarBytes);
    uint8_t *xs = ring + p.stages * p.slot_bytes + kBarBytes + kRedBytes;

    const int tid = threadIdx.x, warp = tid >> 5;
    const int region = blockIdx.x / p.ctas_per_region;
    const int cr = blockIdx.x - region * p.ctas_per_region;
    const int g0 = static_cast<int>(static_cast<long long>(p.groups_per_region) * cr / p.ctas_per_region);
    const int g1 = static_cast<int>(static_cast<long long>(p.groups_per_region) * (cr + 1) / p.ctas_per_region);

    if (tid == 0) {
        s_abort = 0;
        prefetch_tmap(&p.tmap[region]);
        for (int s = 0; s < p.stages; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    const uint64_t policy = make_policy(p.l2_policy);

    // Weights do not depend on the previous kernel: start streaming them
    // before waiting on it. Every CTA of this grid is resident here, so the
    // next kernel in the stream may launch now (programmatic dependent launch).
    if (tid == 0) {
        const int nst = (g1 - g0) * p.slices;
        const int first = nst < p.stages ? nst : p.stages;
        for (int s = 0; s < first; ++s) issue_stage<LAYOUT>(p, bars, ring, region, g0, s, policy);
    }
    pdl_launch_dependents();
    pdl_wait_prior_grid();

    // One thread per x block: 256 threads >= 8192 / 32 blocks.
    static_assert(kThreads >= kMaxK / kQK, "stage_x needs a thread per x block");
    stage_x<XMODE>(p.x, p.k, p.round_mode, xs);
    __syncthreads();

    switch (warp) {
        case 0: gemv_body<LAYOUT, 0>(p, bars, red, xs, ring, region, g0, g1, policy, &s_abort); break;
        case 1: gemv_body<LAYOUT, 1>(p, bars, red, xs, ring, region, g0, g1, policy, &s_abort); break;
        case 2: gemv_body<LAYOUT, 2>(p, bars, red, xs, ring, region, g0, g1, policy, &s_abort); break;
        case 3: gemv_body<LAYOUT, 3>(p, bars, red, xs, ring, region, g0, g1, policy, &s_abort); break;
        case 4: gemv_body<LAYOUT, 4>(p, bars, red, xs, ring, region, g0, g1, policy, &s_abort); break;
        case 5: gemv_body<LAYOUT, 5>(p, bars, red, xs, ring, region, g0, g1, policy, &s_abort); break;
        case 6: gemv_body<LAYOUT, 6>(p, bars, red, xs, ring, region, g0, g1, policy, &s_abort); break;
        default: gemv_body<LAYOUT, 7>(p, bars, red, xs, ring, region, g0, g1, policy, &s_abort); break;
    }
}

// x float32[k] -> int8[k] then float32[k/32]; one thread per block.
__global__ void __launch_bounds__(128) q8_quantize_kernel(const float *__restrict__ x, uint8_t *__restrict__ out,
                                                          int k, int round_mode) {
    pdl_launch_dependents();
    pdl_wait_prior_grid();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= k / kQK) return;
    float4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __ldg(reinterpret_cast<const float4 *>(x) + 8 * b + j);
    uint32_t q[8];
    float d;
    (void)q8_quant_block(v, round_mode, q, &d);
    reinterpret_cast<uint4 *>(out)[2 * b] = make_uint4(q[0], q[1], q[2], q[3]);
    reinterpret_cast<uint4 *>(out)[2 * b + 1] = make_uint4(q[4], q[5], q[6], q[7]);
    reinterpret_cast<float *>(out + k)[b] = __half2float(__float2half_rn(d));
}

constexpr uint32_t kPrefetchChunk = 32768;

__global__ void l2_prefetch_kernel(const uint8_t *r0, const uint8_t *r1, const uint8_t *r2, const uint8_t *r3,
                                   int nregions, size_t bytes) {
    const uint8_t *regs[4] = {r0, r1, r2, r3};
    const size_t chunks = (bytes + kPrefetchChunk - 1) / kPrefetchChunk;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < chunks * nregions;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int r = static_cast<int>(i / chunks);
        const size_t off = (i % chunks) * kPrefetchChunk;
        const size_t len = (bytes - off < kPrefetchChunk ? bytes - off : kPrefetchChunk) & ~static_cast<size_t>(15);
        if (len) bulk_prefetch_l2(regs[r] + off, static_cast<uint32_t>(len));
    }
}

// ------------------------------------------------------------ dispatch

using KernelFn = void (*)(GemvParams);

KernelFn pick_kernel(int layout, int xmode) {
    if (layout == kLayoutRows) return xmode == kXF32 ? q4_gemv_kernel<kLayoutRows, kXF32> : q4_gemv_kernel<kLayoutRows, kXPacked>;
    return xmode == kXF32 ? q4_gemv_kernel<kLayoutPairs, kXF32> : q4_gemv_kernel<kLayoutPairs, kXPacked>;
}

}  // namespace

constexpr int kMaxDevices = 64;

struct DeviceInfo {
    std::atomic<int> ready{0};  // 1 once the fields below are written (release / acquire)
    int sms = 0;
    int smem_optin = 0;
    unsigned *status = nullptr;
};

// Per-device attributes, read once (launch paths are latency-critical). The
// first call on a device fills its entry under a lock; later calls read it
// after an acquire load of `ready`, so a thread never sees a half-written entry.
static DeviceInfo *device_info() {
    static DeviceInfo info[kMaxDevices];
    static std::mutex fill_mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    DeviceInfo &d = info[dev];
    if (d.ready.load(std::memory_order_acquire)) return &d;
    std::lock_guard<std::mutex> lock(fill_mu);
    if (!d.ready.load(std::memory_order_relaxed)) {
        int sms = 0, smem = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return nullptr;
        if (cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return nullptr;
        void *st = nullptr;
        if (cudaGetSymbolAddress(&st, g_status) != cudaSuccess) return nullptr;
        d.status = static_cast<unsigned *>(st);
        d.smem_optin = smem;
        d.sms = sms;
        d.ready.store(1, std::memory_order_release);
    }
    return &d;
}

int sm_count() {
    const DeviceInfo *d = device_info();
    return d ? d->sms : 0;
}

int max_smem_optin() {
    const DeviceInfo *d = device_info();
    return d ? d->smem_optin : 0;
}

unsigned *status_word() {
    const DeviceInfo *d = device_info();
    return d ? d->status : nullptr;
}

bool ensure_smem(const void *fn, int bytes) {
    struct Entry { const void *fn; int dev; int bytes; };
    static Entry cache[256];
    static int used = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    for (int i = 0; i < used; ++i)
        if (cache[i].fn == fn && cache[i].dev == dev && cache[i].bytes >= bytes) return true;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
    // every kernel asks for the same (largest) shared-memory split of the
    // SM's on-chip memory, so CTAs of consecutive launches can share an SM
    if (cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared) !=
        cudaSuccess)
        return false;
    if (used < 256) cache[used++] = Entry{fn, dev, bytes};
    return true;
}

int resident_ctas(const void *fn, int threads, int smem) {
    struct Entry { const void *fn; int dev; int threads; int smem; int ctas; };
    static Entry cache[512];
    static int used = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 1;
    for (int i = 0; i < used; ++i)
        if (cache[i].fn == fn && cache[i].dev == dev && cache[i].threads == threads && cache[i].smem == smem)
            return cache[i].ctas;
    if (!ensure_smem(fn, smem)) return 1;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads, static_cast<size_t>(smem)) != cudaSuccess || n < 1)
        n = 1;
    if (used < 512) cache[used++] = Entry{fn, dev, threads, smem, n};
    return n;
}

namespace {

struct Plan {
    GemvParams p;
    KernelFn fn;
    int grid;
    int smem;
};

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    }
    return fn;
}

// The weight view the kernel streams: [chunk][row][byte of chunk] (ROWS), or
// [chunk][pair][member][byte of chunk] (PAIRS), box = 32 rows x cps chunks,
// landing in shared memory as [cps][32][144].
int encode_region(CUtensorMap *map, int layout, const uint8_t *base, int rows, int k, int cps) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return kErrCuda;
    const cuuint64_t nch = static_cast<cuuint64_t>(k / 256);
    const cuuint64_t row_bytes = static_cast<cuuint64_t>(k / kQK) * kBlockBytes;
    CUresult r;
    if (layout == kLayoutPairs) {
        const cuuint64_t dims[4] = {kChunkBytes, 2, static_cast<cuuint64_t>(rows / 2), nch};
        const cuuint64_t strides[3] = {kChunkBytes, 2 * row_bytes, 2 * kChunkBytes};
        const cuuint32_t box[4] = {kChunkBytes, 2, kGroupRows / 2, static_cast<cuuint32_t>(cps)};
        const cuuint32_t estr[4] = {1, 1, 1, 1};
        r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<uint8_t *>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
        const cuuint64_t dims[3] = {kChunkBytes, static_cast<cuuint64_t>(rows), nch};
        const cuuint64_t strides[2] = {row_bytes, kChunkBytes};
        const cuuint32_t box[3] = {kChunkBytes, kGroupRows, static_cast<cuuint32_t>(cps)};
        const cuuint32_t estr[3] = {1, 1, 1};
        r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t *>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    return r == CUDA_SUCCESS ? 0 : kErrInval;
}

int make_plan(const GemvLaunch &L, const Tuning &tu, bool encode, Plan *out) {
    const char *why = nullptr;
    if (int rc = gemv_validate(L, &why)) return rc;
    const int nb = L.k / kQK, nch = nb / kLanes;
    const int M = L.layout == kLayoutPairs ? 2 : 1;
    KernelFn fn = pick_kernel(L.layout, L.xmode);
    if (!fn) return kErrInval;
    GemvParams p{};
    p.status = status_word();
    if (!p.status) return kErrNoDev;
    p.y = L.y;
    p.x = L.x;
    p.rows_per_region = L.rows / L.nregions;
    p.units_per_region = p.rows_per_region / M;
    p.k = L.k;
    p.nb = nb;
    p.nch = nch;
    p.round_mode = L.round_mode;
    p.l2_policy = L.l2_policy;
    p.groups_per_region = (p.rows_per_region + kGroupRows - 1) / kGroupRows;
    p.xarea_bytes = round_up(xs_bytes(L.k), 16);
    int cps = tu.stage_bytes / kChunkRowsBytes;
    if (cps < 1) cps = 1;
    if (cps > nch) cps = nch;
    p.cps = cps;
    p.slices = (nch + cps - 1) / cps;
    p.slot_bytes = cps * kChunkRowsBytes;
    p.stages = tu.stages < 1 ? 1 : (tu.stages > kMaxStages ? kMaxStages : tu.stages);
    const int limit = max_smem_optin();
    const int fixed = kSmemAlign + kBarBytes + kRedBytes + p.xarea_bytes;
    while (p.stages > 1 && fixed + p.stages * p.slot_bytes > limit) p.stages -= 1;
    const int smem = fixed + p.stages * p.slot_bytes;
    if (smem > limit) return kErrInval;
    const int sms = sm_count();
    if (sms <= 0) return kErrNoDev;
    int per_sm = tu.ctas_per_sm < 1 ? 1 : tu.ctas_per_sm;
    const int fit = resident_ctas(reinterpret_cast<const void *>(fn), kThreads, smem);
    if (per_sm > fit) per_sm = fit;  // one wave: every CTA resident at once
    const int target = sms * per_sm;
    int cpr = target / L.nregions;
    if (cpr < 1) cpr = 1;
    if (cpr > p.groups_per_region) cpr = p.groups_per_region;
    p.ctas_per_region = cpr;
    if (encode) {
        for (int r = 0; r < L.nregions; ++r)
            if (int rc = encode_region(&p.tmap[r], L.layout, L.region[r], p.rows_per_region, L.k, cps)) return rc;
    }
    out->p = p;
    out->fn = fn;
    out->grid = cpr * L.nregions;
    out->smem = smem;
    return 0;
}

}  // namespace

int gemv_validate(const GemvLaunch &L, const char **why) {
    auto bad = [&](const char *w) { if (why) *why = w; return kErrInval; };
    if (L.nregions != 1 && L.nregions != 4) return bad("nregions must be 1 or 4");
    if (L.layout != kLayoutRows && L.layout != kLayoutPairs) return bad("unknown layout");
    if (L.xmode != kXPacked && L.xmode != kXF32) return bad("unknown x mode");
    if (L.round_mode != kRoundContract && L.round_mode != kRoundRoundf) return bad("unknown rounding mode");
    if (L.k <= 0 || L.k % 256) return bad("k must be a positive multiple of 256 (nb % 8 == 0, q4_0.py:166)");
    if (L.k > kMaxK) return bad("k above 8192");
    if (L.rows <= 0) return bad("rows must be positive");
    if (L.rows % L.nregions) return bad("rows must divide into the regions");
    if (L.layout == kLayoutPairs && (L.nregions != 4 || L.rows % 8)) return bad("gemv2 layout needs 4 regions and rows % 8 == 0");
    for (int r = 0; r < L.nregions; ++r) {
        if (!L.region[r]) return bad("null weight pointer");
        if (reinterpret_cast<uintptr_t>(L.region[r]) % 16) return bad("weight regions must be 16-byte aligned");
    }
    if (!L.x || reinterpret_cast<uintptr_t>(L.x) % 16) return bad("x must be 16-byte aligned");
    if (!L.y || reinterpret_cast<uintptr_t>(L.y) % 4) return bad("y must be 4-byte aligned");
    return 0;
}

int gemv_grid(const GemvLaunch &L, const Tuning &tu, int *grid, int *smem_bytes) {
    Plan pl;
    if (int rc = make_plan(L, tu, false, &pl)) return rc;
    if (grid) *grid = pl.grid;
    if (smem_bytes) *smem_bytes = pl.smem;
    return 0;
}

int gemv_launch(const GemvLaunch &L, const Tuning &tu, cudaStream_t stream) {
    Plan pl;
    if (int rc = make_plan(L, tu, true, &pl)) return rc;
    if (!ensure_smem(reinterpret_cast<const void *>(pl.fn), pl.smem)) return kErrCuda;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(pl.smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = L.pdl ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, pl.fn, pl.p) != cudaSuccess) return kErrCuda;
    return 0;
}

int quantize_launch(const float *x, uint8_t *xpacked, int k, int round_mode, cudaStream_t stream, bool pdl) {
    if (!x || !xpacked || k <= 0 || k % kQK) return kErrInval;
    if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(xpacked) % 16) return kErrInval;
    if (round_mode != kRoundContract && round_mode != kRoundRoundf) return kErrInval;
    const int nb = k / kQK;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((nb + 127) / 128);
    cfg.blockDim = dim3(128);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, q8_quantize_kernel, x, xpacked, k, round_mode) != cudaSuccess) return kErrCuda;
    return 0;
}

int prefetch_l2_launch(const uint8_t *const *region, int nregions, size_t bytes_per_region, cudaStream_t stream) {
    if (nregions < 1 || nregions > 4 || !region) return kErrInval;
    for (int r = 0; r < nregions; ++r)
        if (!region[r] || reinterpret_cast<uintptr_t>(region[r]) % 16) return kErrInval;
    const size_t chunks = (bytes_per_region + kPrefetchChunk - 1) / kPrefetchChunk * nregions;
    int grid = static_cast<int>((chunks + 127) / 128);
    if (grid < 1) grid = 1;
    l2_prefetch_kernel<<<grid, 128, 0, stream>>>(region[0], nregions > 1 ? region[1] : region[0],
                                                  nregions > 2 ? region[2] : region[0],
                                                  nregions > 3 ? region[3] : region[0], nregions, bytes_per_region);
    return cudaGetLastError() == cudaSuccess ? 0 : kErrCuda;
}

int read_status(unsigned *status) {
    if (cudaMemcpyFromSymbol(status, g_status, sizeof(unsigned)) != cudaSuccess) return kErrCuda;
    return 0;
}

int clear_status() {
    const unsigned zero = 0;
    return cudaMemcpyToSymbol(g_status, &zero, sizeof(unsigned)) == cudaSuccess ? 0 : kErrCuda;
}

}  // namespace b200
