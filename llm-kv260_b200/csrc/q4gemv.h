// Internal host-side interface of the Q4_0 x Q8_0 GEMV kernels (not part of
// the C ABI; the entry points in capi.cu call these).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace b200 {

constexpr int kQK = 32;          // weights per block (q4_0.py:59)
constexpr int kBlockBytes = 18;  // fp16 scale + 16 nibble bytes (q4_0.py:60)
constexpr int kLanes = 8;        // q4_0.py:62
constexpr int kChunkBytes = 144; // 8 blocks = 9 x 16 bytes (gemv2_dev.h:61)
constexpr int kMaxK = 8192;      // x held in registers: 8 blocks per thread at most

// Where the weight bytes are and how they are laid out.
//   ROWS:  GGUF row-major Q4_0 rows (gemv_dev.h:19-21), split over 1 or 4
//          regions of rows/nregions rows each (gemv_dev.h:29-35).
//   PAIRS: the gemv2 interleave (gemv2_dev.h:46-49,66-72): 4 regions; inside
//          a region row i pairs with row i + rows/8 and their 144-byte chunks
//          alternate.
enum Layout : int { kLayoutRows = 0, kLayoutPairs = 1 };

// What x is.
//   PACKED: the engine's buffer, int8[k] then float32[k/32] (q4_0.py:193-200).
//   F32:    float32[k], quantised to Q8_0 inside the kernel (q4_0.py:185-188).
enum XMode : int { kXPacked = 0, kXF32 = 1 };

enum RoundMode : int { kRoundContract = 0, kRoundRoundf = 1 };

// L2 policy for the streamed weight bytes.
enum L2Policy : int { kL2EvictFirst = 0, kL2EvictNormal = 1, kL2EvictLast = 2 };

// Device status bits (a word per device, read with read_status()).
enum Status : unsigned { kStatusOk = 0, kStatusStageTimeout = 1u, kStatusPeerTimeout = 2u };

struct GemvLaunch {
    const uint8_t *region[4] = {nullptr, nullptr, nullptr, nullptr};
    int nregions = 1;
    int rows = 0;
    int k = 0;
    int layout = kLayoutRows;
    int xmode = kXPacked;
    const void *x = nullptr;
    float *y = nullptr;
    int round_mode = kRoundContract;
    int l2_policy = kL2EvictFirst;
    bool pdl = false;  // launch with programmatic stream serialisation
};

struct Tuning {
    int stage_bytes = 16384;  // target bytes per pipeline stage
    int stages = 4;           // stages in flight per CTA
    int ctas_per_sm = 2;      // grid = SMs x this, at most one CTA per stage
    int xreg_chunks = 8;      // rows of at most this many 144-byte chunks keep x in registers
    int kslices = 1;          // tile kernel: split each row's chunks over at least this many thread slices (1, 2, 4)
};

// Error codes shared with the C ABI (negative errno values).
constexpr int kErrInval = -22;   // -EINVAL
constexpr int kErrNoDev = -19;   // -ENODEV
constexpr int kErrTimeout = -110;  // -ETIMEDOUT
constexpr int kErrBusy = -16;    // -EBUSY
constexpr int kErrCuda = -5;     // -EIO: a CUDA call failed
constexpr int kErrNoMem = -12;   // -ENOMEM

// Checks shapes and alignment; returns 0 or kErrInval with *why set.
int gemv_validate(const GemvLaunch &L, const char **why);
int gemv_launch(const GemvLaunch &L, const Tuning &tu, cudaStream_t stream);

// x float32[k] -> engine buffer int8[k] + float32[k/32] (quantize_q8_0 + pack_x_for_engine).
int quantize_launch(const float *x, uint8_t *xpacked, int k, int round_mode, cudaStream_t stream, bool pdl);

// Pull `bytes` bytes at each region start into L2 (gemv2's fetch-ahead).
int prefetch_l2_launch(const uint8_t *const *region, int nregions, size_t bytes_per_region, cudaStream_t stream);

// ----------------------------------------------------------- tile layout
// The engine's re-laid weights (see q4tile.cu): rows padded to a multiple of
// kTileRows; tile (group g, chunk c) of kTileBytes at ((g * k/256) + c) * kTileBytes.
constexpr int kTileRows = 16;
constexpr int kTileBytes = kTileRows * kLanes * kBlockBytes;  // 2304

// ----------------------------------------------------------- decoder ops
// What the decoder (decoder.cu) fuses into a tile GEMV, around the block dots.
//
// Prologue: how the CTA makes its float32 x before quantising it.
enum Prologue : int {
    kProPlain = 0,      // x as given
    kProRmsnorm = 1,    // x = rmsnorm(res) * norm_w (tp_llama.cpp:557-569)
    kProEmbedNorm = 2,  // res = embed(tokens[*pos]) (tp_llama.cpp:593-604, CTA 0 writes it), then as kProRmsnorm
};
// Epilogue: what happens to each finished row value v.
enum Epilogue : int {
    kEpiStore = 0,      // y[row] = v
    kEpiRopeKv = 1,     // q|k|v rows: rope q and k (tp_llama.cpp:581-591), q, k, v -> y, k and v -> the KV cache at *pos
    kEpiSiluPairs = 2,  // rows interleaved gate0, up0, gate1, ...: act[row / 2] = silu(gate) * up (tp_llama.cpp:615-622)
    kEpiResidual = 3,   // res[row] += v with one rank; with several, += the rank-ordered sum of every rank's v
                        // for that row (tp_llama.cpp:515-521 then add_into), exchanged through peer windows
};

constexpr int kMaxDecodeRanks = 8;

// Optional launch trace of the decoder's per-op kernels: thread 0 of CTA b
// (b < kTraceCtas) writes global-timer stamps (ns) at trace[b * 16 + j]:
// 0 after the CTA's set-up, 1 when the previous kernel's results are visible
// (griddepcontrol.wait returned), 2 when its input is staged (attention: p
// computed), 3 at its end; the tile GEMV also 4 its first weight stage
// landed, 5 its row groups done (thread 0's quad), with an RMSNorm prologue
// 6 the sum of squares' warp reduction done and 7 the norm scale known;
// attention 4 q staged,
// 5 scores and maxima, 6 exponentials, 7 sums, 8 + 2c / 9 + 2c V^T chunk c
// (< 4) landed / consumed.
constexpr int kTraceCtas = 1024;
constexpr int kTraceStamps = 16;

struct DecodeOps {
    int pro = kProPlain;
    int epi = kEpiStore;
    float *res = nullptr;              // residual stream x (kProRmsnorm/kProEmbedNorm: [k]; kEpiResidual: [rows])
    const float *norm_w = nullptr;     // RMSNorm weight [k]
    float eps = 0.0f;
    int exact_norm = 0;                // 1: always sum the squares in the reference's order
    const uint8_t *embd = nullptr;     // token_embd, GGUF Q4_0 rows [n_vocab][k/32*18]
    const int *tokens = nullptr;       // token id by position
    int *in_token = nullptr;           // optional (embedding prologue): >= 0 is the token at pos, taken instead
                                       // of tokens[pos] and recorded there by CTA 0
    const int *pos = nullptr;          // the current position (device)
    const float *rope_cs = nullptr;    // [ctx_max][head_dim]: cos, sin of pair i at 2i, 2i+1
    int head_dim = 0, q_rows = 0, kv_rows = 0, ctx_max = 0, kv_f16 = 1;
    int kv_stride = 0;                 // positions per head in the caches (a multiple of 8, >= ctx_max)
    void *kcache = nullptr;            // this layer's K cache [kv head][kv_stride][head_dim]
    void *vcache = nullptr;            // and V^T cache [kv head][head_dim][kv_stride]
    float *act = nullptr;              // kEpiSiluPairs output [rows / 2]
    uint8_t *act_q8 = nullptr;         // kEpiSiluPairs, optional: act also as packed x for the next GEMV --
                                       // int8[rows / 2] then float32 scale per 32 (q4_0.py:193-200); the row
                                       // groups are then split over CTAs in units of 4 (whole 32-value blocks)
    int nranks = 1, rank = 0;          // kEpiResidual across ranks:
    uint64_t *win_words[kMaxDecodeRanks] = {};  // every rank's word area as mapped here, [slot][source rank][row]
    uint64_t slot_words = 0;           // words per (slot, source rank)
    const unsigned *step = nullptr;    // tokens done; epoch = step * ar_per_token + ar_index + 1
    int ar_per_token = 0, ar_index = 0;
    unsigned *peer_status = nullptr;   // bit kStatusPeerTimeout on a wait that ran out
    int *adv_pos = nullptr;            // with a fused pick: after it, the token loop advances (one rank)
    unsigned *adv_step = nullptr;
    int *adv_tokens = nullptr;         // tokens[pos + 1] = the pick when pos + 1 >= *n_prompt
    const int *n_prompt = nullptr;
    int *adv_in_token = nullptr;       // optional: reset to -1 by the advance
    unsigned *adv_status = nullptr;    // optional: [0] the status word, [1] the peer status word (0 without
                                       // one), as the advance sees them
};

struct TileLaunch {
    const uint8_t *w = nullptr;  // tiles
    int rows = 0;
    int k = 0;
    int xmode = kXPacked;
    const void *x = nullptr;
    float *y = nullptr;
    int round_mode = kRoundContract;
    int l2_policy = kL2EvictFirst;
    bool pdl = false;
    // optional fused greedy pick (see argmax_launch for the rule)
    int *sel_out = nullptr;       // 8 bytes: int32 index + sel_base, float32 value
    int sel_base = 0;
    void *sel_scratch = nullptr;  // tile_select_scratch_bytes(), ticket zeroed once
    DecodeOps dec;                // decoder prologue/epilogue (plain GEMV by default)
    uint64_t *trace = nullptr;    // optional: [CTA < kTraceCtas][kTraceStamps] global-timer stamps
    int max_stages = 0;           // > 0: at most this many ring stages (below Tuning::stages)
    // Size the ring to the busiest CTA's row groups (a small ring leaves room
    // on the SM for the next launch's CTA: the decoder's chain of dependent
    // launches). Off, the ring has as many stages as Tuning asks and fit.
    bool ring_to_groups = false;
};
int tile_select_scratch_bytes();

size_t tiled_bytes(int rows, int k);  // 0 for an unusable shape
int tile_validate(const TileLaunch &L, const char **why);
int tile_launch(const TileLaunch &L, const Tuning &tu, cudaStream_t stream);
int tile_grid(const TileLaunch &L, const Tuning &tu, int *grid, int *smem_bytes);
// GGUF Q4_0 rows (2-byte aligned) -> tiles (16-byte aligned, tiled_bytes(rows, k) bytes).
int repack_launch(const uint8_t *src_rows, int rows, int k, uint8_t *dst_tiles, cudaStream_t stream);

// ----------------------------------------------------------- greedy pick
// First index of the largest of y[0..n) (tp_llama.cpp:879-882), plus
// index_base, into *out_index / *out_value. `scratch` holds
// argmax_scratch_bytes() bytes of per-CTA candidates.
constexpr int kArgmaxMaxParts = 1024;
int argmax_scratch_bytes();
int argmax_launch(const float *y, int n, int index_base, void *scratch, int *out_index, float *out_value,
                  cudaStream_t stream, bool pdl);

int read_status(unsigned *status);   // device status word of the current device
// Record `msg` as the calling thread's last error; returns code.
int report_error(int code, const char *msg);
int clear_status();

// Grid the GEMV would launch (for the bench's roofline accounting).
int gemv_grid(const GemvLaunch &L, const Tuning &tu, int *grid, int *smem_bytes);

}  // namespace b200
