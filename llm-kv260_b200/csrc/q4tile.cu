// Q4_0 x Q8_0 GEMV over the B200 tile layout: the engine path's kernel.
// Bit-exact to src/llm_kv260/q4_0.py:151-182, like the GGUF-layout kernel in
// q4gemv.cu; only where the bytes sit differs.
//
// Tile layout. The reference re-lays every matrix at load for its engine
// (board/tp/tp_llama.cpp:102-118, the gemv2 chunk interleave); this engine
// does the same for HBM. Rows are padded to a multiple of 16. For row group
// g (rows 16g..16g+15) and chunk c (blocks 8c..8c+7) a 2304-byte tile sits at
// byte ((g * nch) + c) * 2304:
//     [0, 2048)     nibbles: 16 bytes for lane l, row i at (l * 16 + i) * 16
//     [2048, 2304)  scales:  float16 bits for lane l, row i at 2048 + (l * 16 + i) * 2
// The 16 nibble bytes of a block are copied unchanged (byte j: weight j in
// the low nibble, weight j+16 in the high one), so the bytes per weight stay
// 18/32 and the algorithmic traffic is the GGUF file's.
//
// Kernel. 128 threads: thread t owns lane L = t / 16 (blocks 8c + L) of row
// i = t % 16 and runs that lane's sequential float32 chain. A stage is a run
// of whole tiles of one row group, moved by ONE 1-D bulk copy (TMA engine,
// no multicast) into an mbarrier ring. Every block is one conflict-free
// 128-bit shared load (a warp reads 512 contiguous bytes) plus a 16-bit
// scale load, 8 __dp4a, two rounded multiplies and the lane add; all warps run
// identical code. Per row group the 8 lane sums meet in tree_sum's order
// through shared memory.
#include <cuda_fp16.h>

#include "common.cuh"

namespace b200 {

namespace {

constexpr int kTileThreads = kTileRows * kLanes;   // 128
constexpr int kTileNibBytes = kTileThreads * 16;   // 2048
constexpr int kMaxStages = 8;
constexpr int kBarBytes = 64;
constexpr int kRedBytes = 2 * kTileThreads * 4;    // double-buffered lane sums
constexpr int kSmemAlign = 128;
constexpr int kXRegMaxChunks = 8;                  // x in registers up to K = 2048

struct TileParams {
    const uint8_t *w;
    float *y;
    const void *x;
    unsigned *status;
    int rows, k, nb, nch;
    int groups;
    int cps;         // tiles (chunks) per stage
    int slices;      // stages per row group
    int slot_bytes;  // cps * 2304
    int stages;
    int round_mode;
    int l2_policy;
};

__device__ __forceinline__ void issue_tile_stage(const TileParams &p, uint64_t *bars, uint8_t *ring, int g0, int s,
                                                 uint64_t policy) {
    const int g = g0 + s / p.slices, c0 = (s % p.slices) * p.cps;
    const int cc = min(p.cps, p.nch - c0);
    const int slot = s % p.stages;
    const uint32_t bytes = static_cast<uint32_t>(cc * kTileBytes);
    mbar_arrive_expect_tx(&bars[slot], bytes);
    bulk_g2s(ring + slot * p.slot_bytes, p.w + (static_cast<size_t>(g) * p.nch + c0) * kTileBytes, bytes, &bars[slot],
             policy);
}

// NCH > 0: x in registers and a stage holds whole rows (K = 256 * NCH).
// NCH == 0: x read per block from shared memory, stages of p.cps tiles.
template <int XMODE, int NCH>
__global__ void __launch_bounds__(kTileThreads) q4_tile_kernel(const __grid_constant__ TileParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ int s_abort;
    uint8_t *ring = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + kSmemAlign - 1) & ~static_cast<uintptr_t>(kSmemAlign - 1));
    uint64_t *bars = reinterpret_cast<uint64_t *>(ring + p.stages * p.slot_bytes);
    float *red = reinterpret_cast<float *>(ring + p.stages * p.slot_bytes + kBarBytes);
    uint8_t *xs = ring + p.stages * p.slot_bytes + kBarBytes + kRedBytes;

    const int t = threadIdx.x, L = t / kTileRows;
    const int g0 = static_cast<int>(static_cast<long long>(p.groups) * blockIdx.x / gridDim.x);
    const int g1 = static_cast<int>(static_cast<long long>(p.groups) * (blockIdx.x + 1) / gridDim.x);
    const int S = p.stages;
    const int nst = (g1 - g0) * p.slices;

    if (t == 0) {
        s_abort = 0;
        for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    const uint64_t policy = make_policy(p.l2_policy);
    // The weights do not depend on the previous kernel: start them moving,
    // let the next kernel launch, then wait for x.
    if (t == 0)
        for (int s = 0; s < nst && s < S; ++s) issue_tile_stage(p, bars, ring, g0, s, policy);
    pdl_launch_dependents();
    pdl_wait_prior_grid();

    stage_x<XMODE>(p.x, p.k, p.round_mode, xs);
    __syncthreads();
    XBlock xr[NCH > 0 ? NCH : 1];
    if constexpr (NCH > 0) {
#pragma unroll
        for (int c = 0; c < NCH; ++c) load_xblock_smem(xs, p.k, 8 * c + L, xr[c]);
    }

    float acc = 0.0f;
    int s = 0;
    for (; s < nst; ++s) {
        const int slot = s % S, gi = s / p.slices, sl = s % p.slices;
        if (!wait_stage(&bars[slot], static_cast<uint32_t>((s / S) & 1), p.status)) s_abort = 1;
        const uint8_t *tile = ring + slot * p.slot_bytes;
        if constexpr (NCH > 0) {
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
                const uint4 nv = *reinterpret_cast<const uint4 *>(tile + c * kTileBytes + t * 16);
                const uint32_t db = *reinterpret_cast<const uint16_t *>(tile + c * kTileBytes + kTileNibBytes + t * 2);
                const uint32_t n[4] = {nv.x, nv.y, nv.z, nv.w};
                acc = __fadd_rn(acc, block_term_words(n, db, xr[c]));
            }
        } else {
            const int c0 = sl * p.cps, cc = min(p.cps, p.nch - c0);
#pragma unroll 2
            for (int j = 0; j < cc; ++j) {
                const uint4 nv = *reinterpret_cast<const uint4 *>(tile + j * kTileBytes + t * 16);
                const uint32_t db = *reinterpret_cast<const uint16_t *>(tile + j * kTileBytes + kTileNibBytes + t * 2);
                const uint32_t n[4] = {nv.x, nv.y, nv.z, nv.w};
                XBlock xb;
                load_xblock_smem(xs, p.k, 8 * (c0 + j) + L, xb);
                acc = __fadd_rn(acc, block_term_words(n, db, xb));
            }
        }
        const bool last_slice = sl == p.slices - 1;
        float *rbuf = red + (gi & 1) * kTileThreads;
        if (last_slice) {
            rbuf[t] = acc;  // [lane][row]
            acc = 0.0f;
        }
        __syncthreads();
        if (s_abort) break;
        if (t == 0 && s + S < nst) issue_tile_stage(p, bars, ring, g0, s + S, policy);
        if (last_slice && t < kTileRows) {
            const float *r = rbuf + t;
            const float yv = tree8(r[0 * kTileRows], r[1 * kTileRows], r[2 * kTileRows], r[3 * kTileRows],
                                   r[4 * kTileRows], r[5 * kTileRows], r[6 * kTileRows], r[7 * kTileRows]);
            const int row = (g0 + gi) * kTileRows + t;
            if (row < p.rows) p.y[row] = yv;
        }
    }
    if (s < nst && t == 0) {
        // Aborted on a stage timeout: let copies already in flight land (each
        // wait bounded) before the CTA's shared memory goes away.
        for (int r = s; r < nst && r < s + S; ++r) (void)wait_stage(&bars[r % S], static_cast<uint32_t>((r / S) & 1), p.status);
    }
}

// GGUF rows -> tiles; one thread per (row, block), padded rows become zeros.
__global__ void repack_tiles_kernel(const uint8_t *__restrict__ src, int rows, int k, uint8_t *__restrict__ dst) {
    const int nb = k / kQK, nch = nb / kLanes;
    const long long total = static_cast<long long>((rows + kTileRows - 1) / kTileRows) * kTileRows * nb;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int r = static_cast<int>(idx / nb), b = static_cast<int>(idx % nb);
        uint16_t h[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
        if (r < rows) {
            const uint16_t *blk = reinterpret_cast<const uint16_t *>(src + (static_cast<size_t>(r) * nb + b) * kBlockBytes);
#pragma unroll
            for (int j = 0; j < 9; ++j) h[j] = blk[j];
        }
        const int g = r / kTileRows, i = r % kTileRows, c = b / kLanes, l = b % kLanes;
        uint8_t *tile = dst + (static_cast<size_t>(g) * nch + c) * kTileBytes;
        uint4 nv;
        nv.x = h[1] | (static_cast<uint32_t>(h[2]) << 16);
        nv.y = h[3] | (static_cast<uint32_t>(h[4]) << 16);
        nv.z = h[5] | (static_cast<uint32_t>(h[6]) << 16);
        nv.w = h[7] | (static_cast<uint32_t>(h[8]) << 16);
        *reinterpret_cast<uint4 *>(tile + (l * kTileRows + i) * 16) = nv;
        *reinterpret_cast<uint16_t *>(tile + kTileNibBytes + (l * kTileRows + i) * 2) = h[0];
    }
}

using TileKernelFn = void (*)(TileParams);

template <int XMODE>
TileKernelFn pick_tile(int nch_reg) {
    switch (nch_reg) {
        case 1: return q4_tile_kernel<XMODE, 1>;
        case 2: return q4_tile_kernel<XMODE, 2>;
        case 3: return q4_tile_kernel<XMODE, 3>;
        case 4: return q4_tile_kernel<XMODE, 4>;
        case 5: return q4_tile_kernel<XMODE, 5>;
        case 6: return q4_tile_kernel<XMODE, 6>;
        case 7: return q4_tile_kernel<XMODE, 7>;
        case 8: return q4_tile_kernel<XMODE, 8>;
        default: return q4_tile_kernel<XMODE, 0>;
    }
}

struct TilePlan {
    TileParams p;
    TileKernelFn fn;
    int grid;
    int smem;
};

int make_tile_plan(const TileLaunch &L, const Tuning &tu, TilePlan *out) {
    const char *why = nullptr;
    if (int rc = tile_validate(L, &why)) return rc;
    const int nb = L.k / kQK, nch = nb / kLanes;
    const bool xreg = nch <= tu.xreg_chunks && nch <= kXRegMaxChunks;
    TileKernelFn fn = L.xmode == kXF32 ? pick_tile<kXF32>(xreg ? nch : 0) : pick_tile<kXPacked>(xreg ? nch : 0);
    TileParams p{};
    p.w = L.w;
    p.y = L.y;
    p.x = L.x;
    p.status = status_word();
    if (!p.status) return kErrNoDev;
    p.rows = L.rows;
    p.k = L.k;
    p.nb = nb;
    p.nch = nch;
    p.groups = (L.rows + kTileRows - 1) / kTileRows;
    int cps = xreg ? nch : tu.stage_bytes / kTileBytes;
    if (cps < 1) cps = 1;
    if (cps > nch) cps = nch;
    p.cps = cps;
    p.slices = (nch + cps - 1) / cps;
    p.slot_bytes = cps * kTileBytes;
    p.stages = tu.stages < 1 ? 1 : (tu.stages > kMaxStages ? kMaxStages : tu.stages);
    p.round_mode = L.round_mode;
    p.l2_policy = L.l2_policy;
    const int xarea = round_up(L.k + 8 * nb, 16);
    const int fixed = kSmemAlign + kBarBytes + kRedBytes + xarea;
    const int limit = max_smem_optin();
    while (p.stages > 1 && fixed + p.stages * p.slot_bytes > limit) p.stages -= 1;
    const int smem = fixed + p.stages * p.slot_bytes;
    if (smem > limit) return kErrInval;
    const int sms = sm_count();
    if (sms <= 0) return kErrNoDev;
    int per_sm = tu.ctas_per_sm < 1 ? 1 : tu.ctas_per_sm;
    const int fit = resident_ctas(reinterpret_cast<const void *>(fn), kTileThreads, smem);
    if (per_sm > fit) per_sm = fit;  // one wave: every CTA resident at once
    int grid = sms * per_sm;
    if (grid > p.groups) grid = p.groups;
    out->p = p;
    out->fn = fn;
    out->grid = grid;
    out->smem = smem;
    return 0;
}

}  // namespace

size_t tiled_bytes(int rows, int k) {
    if (rows <= 0 || k <= 0 || k % 256) return 0;
    return static_cast<size_t>((rows + kTileRows - 1) / kTileRows) * (k / 256) * kTileBytes;
}

int tile_validate(const TileLaunch &L, const char **why) {
    auto bad = [&](const char *w) { if (why) *why = w; return kErrInval; };
    if (L.xmode != kXPacked && L.xmode != kXF32) return bad("unknown x mode");
    if (L.round_mode != kRoundContract && L.round_mode != kRoundRoundf) return bad("unknown rounding mode");
    if (L.k <= 0 || L.k % 256) return bad("k must be a positive multiple of 256 (nb % 8 == 0, q4_0.py:166)");
    if (L.k > kMaxK) return bad("k above 8192");
    if (L.rows <= 0) return bad("rows must be positive");
    if (!L.w || reinterpret_cast<uintptr_t>(L.w) % 16) return bad("tiles must be 16-byte aligned");
    if (!L.x || reinterpret_cast<uintptr_t>(L.x) % 16) return bad("x must be 16-byte aligned");
    if (!L.y || reinterpret_cast<uintptr_t>(L.y) % 4) return bad("y must be 4-byte aligned");
    return 0;
}

int tile_grid(const TileLaunch &L, const Tuning &tu, int *grid, int *smem_bytes) {
    TilePlan pl;
    if (int rc = make_tile_plan(L, tu, &pl)) return rc;
    if (grid) *grid = pl.grid;
    if (smem_bytes) *smem_bytes = pl.smem;
    return 0;
}

int tile_launch(const TileLaunch &L, const Tuning &tu, cudaStream_t stream) {
    TilePlan pl;
    if (int rc = make_tile_plan(L, tu, &pl)) return rc;
    if (!ensure_smem(reinterpret_cast<const void *>(pl.fn), pl.smem)) return kErrCuda;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(kTileThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(pl.smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = L.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, pl.fn, pl.p) == cudaSuccess ? 0 : kErrCuda;
}

int repack_launch(const uint8_t *src_rows, int rows, int k, uint8_t *dst_tiles, cudaStream_t stream) {
    if (!src_rows || !dst_tiles || rows <= 0 || k <= 0 || k % 256) return kErrInval;
    if (reinterpret_cast<uintptr_t>(src_rows) % 2 || reinterpret_cast<uintptr_t>(dst_tiles) % 16) return kErrInval;
    const long long total = static_cast<long long>((rows + kTileRows - 1) / kTileRows) * kTileRows * (k / kQK);
    long long blocks = (total + 255) / 256;
    if (blocks > 65535LL * 16) blocks = 65535LL * 16;
    repack_tiles_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(src_rows, rows, k, dst_tiles);
    return cudaGetLastError() == cudaSuccess ? 0 : kErrCuda;
}

}  // namespace b200
