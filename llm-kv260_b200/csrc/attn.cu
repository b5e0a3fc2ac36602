// Decode attention for one layer, bit-exact to the reference runtime's
// attention_group (board/tp/tp_llama.cpp:644-690) over this rank's heads:
// one CTA of kAttnThreads per local KV head running attn_core (attn_core.cuh,
// which states the order of every operation).
//
// Before the kernel waits for its predecessor (the q|k|v GEMV that writes
// this position's K row and V column), the last warp asks L2 for the head's K rows
// and V^T columns of the positions before it -- written by earlier tokens --
// so the loads after the wait hit L2. The prefetch is a hint sized from a
// read of the position that may be one token stale; what is read after the
// wait is the current data either way (L2 is the point of coherence).
#include <cuda_fp16.h>

#include "attn_core.cuh"
#include "common.cuh"
#include "decode.h"

namespace b200 {

namespace {

constexpr int kAttnThreads = 256;

// V^T bytes per column per chunk, and K rows per chunk (64 KB of K)
__host__ __device__ constexpr int attn_colb(int d) { return d == 64 ? 512 : 256; }
__host__ __device__ constexpr int attn_kc(int d, int esz) { return 65536 / (d * esz); }

struct AttnParams {
    const float *q;
    const uint8_t *kcache, *vcache;  // this layer: K [kv head][stride][D], V^T [kv head][D][stride]
    float *out;
    const int *pos;
    unsigned *status;
    int group, stride, ctx_max;
    float scale;
    uint64_t *trace;  // optional launch trace (q4gemv.h, kTraceCtas)
};

__device__ __forceinline__ uint64_t *attn_rec(uint64_t *trace) {
    return (trace && blockIdx.x < kTraceCtas) ? trace + blockIdx.x * kTraceStamps : nullptr;
}

template <int D, int ESZ>
__global__ void __launch_bounds__(kAttnThreads, 1) attn_kernel(const __grid_constant__ AttnParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t bars[kAttnBars];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    const int kvh = blockIdx.x, G = p.group;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kAttnBars; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    const size_t head_bytes = static_cast<size_t>(p.stride) * D * ESZ;
    const uint8_t *kb = p.kcache + kvh * head_bytes;
    const uint8_t *vtb = p.vcache + kvh * head_bytes;
    uint64_t *rec = attn_rec(p.trace);
    pdl_launch_dependents();
    attn_stamp_at(rec, 0);
    if (threadIdx.x >= kAttnThreads - 32) {  // the last warp: thread 0's warp goes straight to the wait
        const int hint = *reinterpret_cast<const volatile int *>(p.pos) + 2;  // may be a token behind: a hint
        attn_prefetch_l2<D, ESZ>(kb, vtb, p.stride, hint < 1 ? 1 : (hint > p.ctx_max ? p.ctx_max : hint));
    }
    pdl_wait_prior_grid();
    attn_stamp_at(rec, 1);
    const int n = *p.pos + 1;
    uint32_t par = 0;
    (void)attn_core<D, ESZ, attn_colb(D), attn_kc(D, ESZ), kAttnThreads>(
        p.q + static_cast<size_t>(kvh) * G * D, kb, vtb, p.stride, n, G, p.scale,
        p.out + static_cast<size_t>(kvh) * G * D, smem, 1, bars, par, p.status, rec);
    if (rec) {
        named_sync(1, kAttnThreads);
        attn_stamp_at(rec, 3);
    }
}

using AttnFn = void (*)(AttnParams);

AttnFn pick_attn(int d, int kv_f16) {
    if (d == 64) return kv_f16 ? attn_kernel<64, 2> : attn_kernel<64, 4>;
    if (d == 128) return kv_f16 ? attn_kernel<128, 2> : attn_kernel<128, 4>;
    return nullptr;
}

}  // namespace

int attn_kv_stride(int ctx_max) { return (ctx_max + 7) / 8 * 8; }

int attn_smem_bytes(int head_dim, int kv_f16, int ctx_max) {
    const int esz = kv_f16 ? 2 : 4;
    return 128 + attn_core_smem_bytes(head_dim, esz, attn_colb(head_dim), attn_kc(head_dim, esz), kAttnThreads,
                                      attn_kv_stride(ctx_max));
}

int attn_launch(const AttnLaunch &L, cudaStream_t stream) {
    AttnFn fn = pick_attn(L.head_dim, L.kv_f16);
    if (!fn) return kErrInval;
    if (L.group < 1 || L.group > 4 || L.kvh_local < 1 || L.ctx_max < 1 || L.kv_stride != attn_kv_stride(L.ctx_max))
        return kErrInval;
    if (!L.q || !L.kcache || !L.vcache || !L.out || !L.pos) return kErrInval;
    if (reinterpret_cast<uintptr_t>(L.kcache) % 16 || reinterpret_cast<uintptr_t>(L.vcache) % 16) return kErrInval;
    const int smem = attn_smem_bytes(L.head_dim, L.kv_f16, L.ctx_max);
    if (smem > max_smem_optin()) return kErrInval;
    if (!ensure_smem(reinterpret_cast<const void *>(fn), smem)) return kErrCuda;
    AttnParams p{};
    p.q = L.q;
    p.kcache = static_cast<const uint8_t *>(L.kcache);
    p.vcache = static_cast<const uint8_t *>(L.vcache);
    p.out = L.out;
    p.pos = L.pos;
    p.status = status_word();
    if (!p.status) return kErrNoDev;
    p.group = L.group;
    p.stride = L.kv_stride;
    p.ctx_max = L.ctx_max;
    p.scale = L.scale;
    p.trace = L.trace;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(L.kvh_local);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = L.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, fn, p) == cudaSuccess ? 0 : kErrCuda;
}

}  // namespace b200
