// The persistent decode step (step.cu): every kernel of a decode step as
// phases of one cooperative launch.
#pragma once
#include "decode.cuh"

namespace reng {

constexpr int kStepWarps = 8;        // warps per CTA (one CTA per SM)
constexpr int kStepChunk = 8192;     // bytes per ring slot (4 bf16 / 8 FP8 packed blocks)
constexpr int kStepMaxStages = 4;    // ring slots per warp
constexpr int kStepAttnKeys = 32;    // keys per attention sub-chunk (a lane per key)
constexpr int kAttnMaxHpgStep = 8;   // query heads per KV head the step kernel supports

enum StepPhaseKind : int { PH_EMBED = 0, PH_GEMV = 1, PH_ATTN = 2 };

struct StepPhase {
    int kind;
    int epi;             // PH_GEMV: the epilogue
    long long blocks;    // PH_GEMV: tiles * kc packed blocks, split evenly over the CTAs
    int slots;           // PH_GEMV: most CTAs sharing one tile
    union {
        GemvArgs g;      // PH_GEMV (its x, norm, outputs; g.M rows)
        AttnArgs at;     // PH_ATTN
        EmbedArgs em;    // PH_EMBED
    };
};

// The weight-chunk sequence of a phase (kept in shared memory by the kernel).
struct StepSeq {
    const uint8_t* w;   // packed weights (null: not a GEMV phase)
    int blocks;         // tiles * kc
    short kc;           // blocks per tile
    short bb;           // bytes per block
};

struct StepCtl {
    const StepPhase* ph;
    const StepSeq* seq;      // [nph]
    int nph;
    int stages;              // ring slots per warp
    int xbytes;              // shared x / attention scratch bytes
    int attn_units;          // most units (key ranges) per (row, KV group)
    float4* part;            // cross-CTA tile partials [tile][slot][32 lanes]
    unsigned int* tile_cnt;  // [tiles] arrivals
    float* apart;            // attention partials [row][group][unit][step_attn_part_len]
    unsigned int* acnt;      // [row][group] arrivals
    unsigned long long* bar; // grid barrier arrivals (grows by the grid per barrier)
    int* abort;              // set when a wait ran out: later barriers fall through
    int* err;
    float* am_val;           // LM head: per-warp argmax partials [G][kMaxRows]
    int* am_idx;
    unsigned int* am_count;
    // phase timeline (null: off): [phase][kTraceStride] = release of the
    // barrier before the phase (seen by CTA 0), earliest and latest CTA
    // arrival at the barrier after it, and for CTA 0 of a projection phase
    // when its x rows were staged and when its last warp left the weight
    // loop; %globaltimer ns
    unsigned long long* trace;
};
constexpr int kTraceStride = 5;

// Floats of one attention unit's partial: o [hpg][hd], max [hpg], sum [hpg],
// padded to 16 bytes.
__host__ __device__ __forceinline__ int step_attn_part_len(int hpg, int hd) { return (hpg * (hd + 2) + 3) & ~3; }
size_t step_attn_smem_bytes();
// Shared bytes of the per-tile reduction of the warps' accumulators (lanes
// q < ceil(M / 2) carry the M activation columns).
__host__ __device__ __forceinline__ int step_red_bytes(int M) { return kStepWarps * 8 * ((M + 1) / 2) * 16; }
// Row stride (elements) of the step kernel's shared x rows: K padded to the
// packed blocks' 64 and 32 elements more (rows 64 bytes apart mod 128).
__host__ __device__ __forceinline__ int step_xstride(int K) { return (K + 63) / 64 * 64 + 32; }
size_t step_smem_bytes(int stages, int xbytes, int nph);
// CTAs per SM the step kernel can keep resident with this shared memory
// (0: does not fit).
int step_blocks_per_sm(int w8, int stages, int xbytes, int nph);
cudaError_t launch_step(const StepCtl& c, int w8, int grid, cudaStream_t st);

}  // namespace reng
