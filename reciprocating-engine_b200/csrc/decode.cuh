// Kernel interfaces of the decode step (see decode.cu for the kernels).
#pragma once
#include "common.cuh"

namespace reng {

// Packed weights.  A block covers 16 rows x 64 k of a projection.
//  * bf16 (2 KB): two 8-row atoms (rows 0-7, rows 8-15), each 8 rows x
//    128 B with the 16-byte chunk j of row r stored at chunk position j ^ r
//    (the K-major 128-byte-swizzle atom of the tcgen05 UMMA operand layout;
//    the XOR also makes the GEMV's 16-byte fragment reads bank-conflict
//    free).  The GEMV lane (g, q) multiplies row g and g+8 at
//    k = 32h + 8q .. +8 for h = 0, 1.
//  * FP8-E4M3 codes (1 KB): half h (512 B) holds rows 8h..8h+7; lane l's
//    16 bytes (offset h*512 + l*16) are row 8h + l/4, k = 16(l%4) .. +16.
// Block (tile, c) of a [tiles x kc] matrix starts at (tile * kc + c) * block
// bytes; a warp's k-range of a tile is contiguous.
constexpr int kTileRows = 16;
constexpr int kChunkK = 64;                 // k per block
constexpr int kBlockBytesBf16 = 2048;
constexpr int kBlockBytesFp8 = 1024;
constexpr int kMaxRows = 8;    // activation rows per GEMV launch (mma N)
constexpr int kRowsCap = 256;  // decode slots of a step; the tcgen05 GEMM's N-tile
constexpr int kBlockRows = 1024;  // rows of a prefill block (work buffers)
constexpr size_t kGemvMaxSmem = 96 * 1024;  // x rows staged in shared memory up to this
// RMS partials ss[m][tile] (sum of squares of 16 residual values), row
// stride kSsStride: a row's partials are contiguous, so the kernels that
// normalise read a few cache lines per row (hidden <= 16 * kSsStride)
constexpr int kSsStride = 512;

// Row stride (elements) of the shared x copy: 32 elements of padding put
// consecutive rows 64 bytes apart, so the fragment loads of a warp hit 32
// distinct banks.
__host__ __device__ __forceinline__ int gemv_xstride(int K) { return K + 32; }

enum Epi : int {
    EPI_QKV = 0,     // bias + RoPE, q to a buffer, k/v into the KV cache
    EPI_RESID = 1,   // x_res += bf16(acc) (bf16), norm partials of x_res
    EPI_SWIGLU = 2,  // act = silu(gate) * up
    EPI_LOGITS = 3,  // bf16 logits + argmax partials, last CTA picks the ids
    EPI_F32 = 4,     // f32 partial out (tensor-parallel o_proj / down_proj)
};

constexpr int kTpMaxWorld = 8;  // tensor-parallel ranks

// The LM head sharded by vocabulary under tensor parallelism (decode
// steps): every rank streams a contiguous range of the head's rows, and
// the ranks swap their per-row argmax keys.  Key area of a rank (in its
// exported region): [2 parities][kTpMaxWorld sources][kMaxRows][2 words],
// each word (epoch << 32) | 32 bits of the key.
struct HeadXchg {
    unsigned long long* recv[kTpMaxWorld];  // every rank's key area (peer mappings; own at [rank])
    unsigned* epoch;                         // exchanges done by this rank
    int rank, world;
};

struct GemvArgs {
    // weights
    const uint8_t* w;  // packed blocks
    int tiles;         // 16-row tiles
    int kc;            // 32-wide k chunks
    int K;             // input width (x columns used; the packing zero-pads to kc*32)
    int M;             // activation rows (<= kMaxRows)
    // activations x [M][ldx] bf16
    const uint16_t* x;
    int ldx;
    // fused RMSNorm of x: inv[m] = 1/sqrt(sum_t ss_in[m][t] / norm_k + eps),
    // x' = bf16(x * inv * gain).  ss_in == nullptr: x used as is.
    const float* ss_in;
    int ss_tiles;
    const float* gain;
    float eps;
    int norm_k;
    // per-row bookkeeping
    const int* row_slot;
    const int* row_pos;
    // epilogue outputs
    uint16_t* out;     // EPI_QKV: q [M][q_dim]; EPI_RESID: x_res [M][ldo];
                       // EPI_SWIGLU: act [M][ldo]; EPI_LOGITS: logits [M][ldo]
    float* out_f32;    // EPI_F32: [M][ldo]
    int ldo;
    float* ss_out;     // EPI_RESID: norm partials [tiles][kRowsCap]
    const float* bias; // EPI_QKV: [q_dim + 2 kv_dim] (q part pre-scaled) or null
    // EPI_QKV
    int head_dim;
    int q_tiles, k_tiles;  // tile ranges: [0,q) q pairs, [q,q+k) k pairs, rest v
    int n_kv;
    const float* rope_cos;  // [cap][hd]
    const float* rope_sin;
    uint16_t* kcache;       // this layer's [B][n_kv][cap][hd]
    uint16_t* vcache;
    int cap;
    // EPI_LOGITS
    int vocab;
    unsigned long long* am_key;  // [kRowsCap] running maximum of am_pack keys per row, 0 between launches
    unsigned int* am_count;
    int mode;               // 0 decode, 1 prefill
    int slot;               // prefill slot
    int batch;              // decode slots
    int* pos;               // [batch] positions
    int* step;              // decode step counter
    uint32_t* ids_ring;     // [(cap+1)][batch]
    uint32_t* next_id;      // prefill: argmax of the last row
    int* err;               // device error word (RENG_E_TIMEOUT from a bounded wait)
    // FP8-E4M3 weights: blocks hold 16 rows x 64 k of codes; the mma runs in
    // f16 (x staged as f16) and the epilogue multiplies by the row's scale
    int w8;
    const float* wscale;    // [tiles*16] per packed row
    // EPI_LOGITS: global index of the first row of tile 0 (a vocabulary
    // shard), and the key exchange of a sharded head (null: every row here)
    int row0;
    const HeadXchg* hx;
};

// Per-head q/k RMSNorm and RoPE (Qwen3's q_norm / k_norm) of the rows a
// q/k/v launch wrote raw (it rotated with the identity table): q heads in the
// q buffer, K heads at each row's cache position, in place.
struct QkNormArgs {
    uint16_t* q;                 // [M][q_dim]
    uint16_t* kcache;            // this layer's K cache [slot][n_kv][cap][hd]
    const float* qn;             // [hd] q gains, the attention scale folded in
    const float* kn;             // [hd] k gains
    const float* rope_cos;       // [cap][hd] the model's tables
    const float* rope_sin;
    const int* row_slot;
    const int* row_pos;
    int M, nq, n_kv, hd, cap, q_dim;
    float eps;
};

struct AttnArgs {
    const uint16_t* q;      // [M][q_dim]
    const uint16_t* kcache; // this layer [B][n_kv][cap][hd]
    const uint16_t* vcache;
    uint16_t* out;          // [M][q_dim]
    const int* row_slot;
    const int* row_pos;
    int M, n_kv, hpg, hd, cap;
    int contiguous;         // rows are consecutive positions of one slot (a prefill block)
};

struct EmbedArgs {
    const uint16_t* table;  // [vocab][hidden]
    int hidden, vocab;
    uint16_t* x_res;        // [M][hidden]
    float* ss_out;          // [hidden/16][kRowsCap]
    int* row_slot;
    int* row_pos;
    int mode;               // 0 decode: ids from ids_ring[step], rows = slots
    int M;
    const int* pos;
    const int* step;
    const uint32_t* ids_ring;
    const uint32_t* prefill_ids;
    int slot;
    int batch;
    int* err;               // an id outside the vocabulary records RENG_E_INVAL here
};

struct Pack8Args {
    const uint8_t* src;    // codes, row-major [rows][K]
    const int* rowmap;     // [tiles*16] source row per packed row, -1 = zero
    int tiles, K, kc;      // kc = ceil(K / 64)
    uint8_t* dst;
};

struct PackArgs {
    const uint16_t* src;   // row-major [rows][ld]
    int64_t ld;
    const int* rowmap;     // [tiles*16] source row per packed row, -1 = zero
    int tiles, K, kc;
    float scale;           // != 0: rows with rowmap < scale_rows are bf16(w*scale)
    int scale_rows;
    uint8_t* dst;
};

// Argmax over CTAs as one 64-bit atomicMax per row: the high word orders the
// f32 values, the low word is ~index, so among equal values the first index
// wins.  The kernels never take NaN or -inf (the reference's fold starts at
// -inf with a strict '>'); a CTA that took nothing packs (-inf, no index),
// which unpacks to index 0, the reference's answer for such a row.  The
// maximum is the same whatever order the CTAs arrive in.
__device__ __forceinline__ unsigned long long am_pack(float v, int i) {
    // -0 packs as +0: the reference's strict '>' fold treats them as equal,
    // so the first index wins between them
    const uint32_t b = v == 0.f ? 0u : __float_as_uint(v);
    const uint32_t ord = (v != v) ? 0u : ((b & 0x80000000u) ? ~b : (b | 0x80000000u));
    return ((unsigned long long)ord << 32) | (unsigned long long)(0xffffffffu - (uint32_t)i);
}
// The index of a row's maximum key (0 for a row of NaN only, or no key).
__device__ __forceinline__ int am_unpack(unsigned long long key) {
    const uint32_t i = 0xffffffffu - (uint32_t)(key & 0xffffffffu);
    return (key == 0ull || i >= 0x7fffffffu) ? 0 : (int)i;
}

// Launchers (return cudaError of the launch).  `pdl` sets programmatic
// stream serialization so the kernel may start before its predecessor ends.
// max_grid > 0 caps the persistent grid (else all resident CTAs); the grid
// actually launched (tiles split evenly over the CTAs) goes to *grid_out.
cudaError_t launch_gemv(const GemvArgs& a, int epi, int nwarp, int max_grid, bool pdl, cudaStream_t st,
                        int* grid_out = nullptr);
cudaError_t gemv_prepare();
// The 3..8-row GEMV with register x fragments (gemv8.cu): whether it runs a
// projection, its launch, and its shared-memory limits (before capture).
bool gemv8_fits(const GemvArgs& a);
cudaError_t launch_gemv8(const GemvArgs& a, int epi, bool pdl, cudaStream_t st);
cudaError_t gemv8_prepare();
cudaError_t launch_attn(const AttnArgs& a, int chunk, bool pdl, cudaStream_t st);
// Key slices per (row, KV group) of a decode attention launch over `units`
// rows x KV groups (RENG_ATTN_SLICES fixes them).
int attn_slices(long long units);
cudaError_t launch_embed(const EmbedArgs& a, bool pdl, cudaStream_t st);
cudaError_t launch_qk_norm(const QkNormArgs& a, bool pdl, cudaStream_t st);
cudaError_t launch_pack(const PackArgs& a, cudaStream_t st);
cudaError_t launch_pack8(const Pack8Args& a, cudaStream_t st);
cudaError_t launch_gather_scales(const float* src, const int* rowmap, int n, float mul, int mul_rows,
                                 float* dst, cudaStream_t st);
cudaError_t launch_bf16_to_f32(const uint16_t* src, float* dst, int64_t n, cudaStream_t st);

int fp8_quantize_device(const uint16_t* w, int64_t rows, int64_t cols, int fmt, int scaling,
                        float backoff, uint8_t* codes, float* scales, uint32_t* bias_dev,
                        cudaStream_t st);

constexpr int kAttnChunk = 64;    // keys per shared-memory tile
constexpr int kAttnCluster = 8;   // CTAs (key slices) per (row, KV group)

}  // namespace reng
