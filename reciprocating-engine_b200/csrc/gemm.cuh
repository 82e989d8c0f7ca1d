// Interfaces of the tcgen05 GEMM path (gemm.cu): projections of steps with
// more activation rows than the GEMV's mma N (batch > 8 decode, prefill).
#pragma once
#include <cuda.h>

#include "decode.cuh"

namespace reng {

constexpr int kGemmRowsPerCta = 128;  // weight rows per CTA (the MMA's M)
constexpr int kGemmMaxSplits = 8;     // K splits of a super-tile (a portable cluster)
constexpr int kGemmCntMax = 1024;     // super-tiles of a split launch (arrival counts)
constexpr int kGemmRowsMax = kBlockRows;  // activation rows of a launch (N-tiles of kRowsCap)
static_assert(kGemmRowsMax <= 4 * kRowsCap, "the LM head's argmax scratch holds 4 * kRowsCap rows");

struct GemmArgs {
    GemvArgs e;               // epilogue arguments (M, outputs, RoPE, cache, argmax ...)
    const uint8_t* w;         // packed bf16 blocks [tiles16][kc]
    int tiles16;              // 16-row tiles of the matrix
    int kc;                   // 64-k chunks
    int super_tiles;          // ceil(tiles16 / 8): 128-row CTA tiles
    int ks;                   // K splits (every split gets >= 1 chunk): one cluster per super-tile
    int N;                    // MMA N: activation rows rounded up to 16 (16..256), kRowsCap when ntiles > 1
    int ntiles;               // N-tiles: CTA (super-tile, N-tile) multiplies activation rows nt*N .. +N
    int stages;               // pipeline stages (2..8)
    int C;                    // 64-k chunks per stage (one weight copy, one activation copy)
    int b3d;                  // the activation map is 3-D ({64, N, C} boxes; K % 64 == 0), else 2-D per chunk
    // ks > 1 without a cluster: f32 partials [super_tiles][ks][128][N] and
    // one arrival count per super-tile (0 between launches); null: the
    // splits form a cluster and add their partials over shared memory
    float* gpart;
    int* gcnt;
};

// Tensor map of a row-major bf16 activation buffer [rows][K] read as
// {64 k, n rows} boxes with the 128-byte swizzle; k >= K reads zeros.
int gemm_tensor_map(const uint16_t* x, int rows, int K, int n, CUtensorMap* out);
// The same buffer as {64 k, n rows, c chunks} boxes (K % 64 == 0).
int gemm_tensor_map3(const uint16_t* x, int rows, int K, int n, int c, CUtensorMap* out);
// Packed bf16 weights [tiles16][kc][2 KB] as {64, 16, 8 tiles, c chunks} boxes.
int gemm_weight_map(const uint8_t* w, int tiles16, int kc, int c, CUtensorMap* out);
size_t gemm_smem_bytes(int n, int stages, int c, bool w8);
// Packed FP8-E4M3 weights [tiles16][kc][1 KB] (row r of a block at r * 64
// bytes) as {64 bytes, 16 rows, 8 tiles, c chunks} boxes, for the GEMM's
// weight-only FP8 path.
int gemm_weight_map8(const uint8_t* w, int tiles16, int kc, int c, CUtensorMap* out);
// A layer's K or V cache as {64, box_rows} boxes of hd-wide rows (128-byte swizzle).
int attn_cache_map(const uint16_t* cache, int hd, long long rows, int box_rows, CUtensorMap* out);
// Prefill-block attention on the tensor cores (attn_prefill.cu): whether a
// block fits it (head_dim 64 or 128, contiguous rows, a cache of cache_rows
// hd-wide rows addressable by 32-bit tensor coordinates) and its launch.
bool attn_prefill_fits(const AttnArgs& a, long long cache_rows);
int launch_attn_prefill(const AttnArgs& a, long long cache_rows, int* err, cudaStream_t st);
// Decode attention with the K/V tiles streamed through a TMA ring
// (attn_decode.cu): whether a launch fits it (head_dim 64 or 128, at most 8
// query heads per group, a cache addressable by 32-bit tensor coordinates)
// and its launch (key slices per row and group as the per-row kernel's).
bool attn_ring_fits(const AttnArgs& a, long long cache_rows);
cudaError_t attn_ring_prepare();  // its shared-memory limit, once per device before capture
int launch_attn_ring(const AttnArgs& a, long long cache_rows, int* err, bool pdl, cudaStream_t st);
// 64-k chunks per pipeline stage.
int gemm_chunks_per_stage(int n);
// Pipeline stages of c chunks for MMA width n: as many as fit two CTAs per
// SM, or at one CTA per SM the bytes in flight of 4 one-chunk stages.
int gemm_pick_stages(int n, bool one_per_sm, int epi, int c, bool w8);
// Raise the dynamic shared-memory limit of every GEMM instantiation (call
// once per device before capture).
cudaError_t gemm_prepare();
// K splits and pipeline stages of a launch over super_tiles x kc blocks.
void gemm_plan(int super_tiles, int kc, int n, int epi, int sms, bool gsplit_ok, int* ks, int* stages, bool* gsplit,
               int* c, bool w8 = false);
cudaError_t launch_gemm_tc(const CUtensorMap& map, const CUtensorMap& wmap, const GemmArgs& g, int epi, bool pdl,
                           cudaStream_t st);
// xn[m] = bf16(x[m] * 1/sqrt(sum_t ss[t][m] / H + eps) * gain), m < M.
cudaError_t launch_rmsnorm_rows(const uint16_t* x, const float* ss, int ss_tiles, const float* gain, float eps,
                                int H, uint16_t* xn, int M, bool pdl, cudaStream_t st);

}  // namespace reng
