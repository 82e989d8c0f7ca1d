// tcgen05 / TMEM GEMM for steps with many activation rows (batch > 8 decode
// and prefill blocks): Y[m, row] = sum_k X[m, k] * W[row, k] with the
// weights as the MMA's A operand (M = 128 weight rows per CTA) and the
// activation rows as its N (16..256), so a wide batch is one N dimension and
// the weights stream from HBM once per step.
//
// Operands in shared memory use the K-major 128-byte-swizzle atom of the
// UMMA descriptors (8 rows x 128 B, 16-byte chunk j of row r at j ^ r):
//  * A (weights): the packed blocks are already that atom; a 4-D tensor map
//    over the packed matrix ({64, 16 rows, tiles, chunks}, no swizzle) lands
//    C chunks x 8 tiles x 2 KB with one copy;
//  * B (activations, row-major [rows][K] bf16): a 3-D tensor-map copy with
//    128-byte swizzle of a {64 k, N rows, C chunks} box (a 2-D copy per
//    chunk when K is not a multiple of 64).
// Both give SBO = 1024 B (one 8-row atom), and the K=16 steps inside a
// 64-k chunk advance the descriptor start address by 32 B.  A stage holds C
// (2) chunks: two copies per 128 KB of weights instead of one per 2 KB
// block, since a single issuing thread's copy count, not the bytes in
// flight, bounded the weight stream (17 GB/s per SM with eight 2 KB copies
// per chunk whatever the stage count, 40 GB/s with one copy per stage,
// B200).
//
// Roles: warp 0 lane 0 issues the copies, warp 1 owns the TMEM accumulator
// (128 lanes x N f32 columns) and lane 0 issues the MMAs and commits each
// stage back to the producer; the epilogue warps 2 .. 2 + 4 W read the
// accumulator with tcgen05.ld (warp w reads TMEM lanes 32*(w%4) .. +32, the
// W warps of a lane quarter every W-th 16-column block) and apply
// the same epilogues as the GEMV kernels.  A weight matrix with few super-tiles
// is split along K over up to 8 CTAs launched as one thread-block cluster:
// each keeps its partial tile in its own shared memory, and after a cluster
// barrier CTA r adds column blocks r, r + ks, ... of every split over
// distributed shared memory in rank order (deterministic) and runs their
// epilogue.  Every mbarrier wait is bounded.
#include <cooperative_groups.h>

#include <mutex>
#include <string>
#include <vector>

#include "gemm.cuh"
#include "gemv_core.cuh"
#include "tc.cuh"

namespace reng {

namespace {

// Epilogue warps per TMEM lane quarter (W, chosen at launch): warp w reads
// lanes 32*(w%4) .. +32, and the W warps of a quarter take every W-th
// 16-column block.  The epilogue of a wide tile is latency-bound (one
// dependent chain per column on each warp), so more warps per quarter drain
// it faster: measured on B200 (Llama-8B widths, 1024-row prefill block)
// gate/up 429 -> 294 us from 1 to 4 warps.  Up to 4 (3 for the q/k/v
// epilogue, whose RoPE operands would spill at the 113 registers of 576
// threads) when N > 64; 1 at N <= 64, where two CTAs share an SM (b64 decode:
// 10.7k tok/s with 1, 9.6k with 4, the SM's registers then holding one).
template <int EPI>
__host__ __device__ constexpr int epi_warps_max() { return EPI == EPI_QKV ? 3 : 4; }
template <int EPI>
__host__ __device__ constexpr int gemm_threads_max() { return 64 + 128 * epi_warps_max<EPI>(); }
constexpr int kGemmMaxStages = 8;  // pipeline stages (runtime: GemmArgs::stages)
constexpr int kGemmStageBudget = 200 * 1024;                  // stage bytes of a one-per-SM launch
constexpr int kGemmMaxDynSmem = kGemmStageBudget + 2048;      // + the 1024-byte alignment slack
constexpr int kStageA = 8 * kBlockBytesBf16;   // 128 rows x 64 k bf16 (the MMA's A operand)
constexpr int kStageA8 = 8 * kBlockBytesFp8;   // the same rows as FP8-E4M3 codes (weight-only FP8)
using namespace tc;

__device__ __forceinline__ void named_sync_epilogue() {
    asm volatile("bar.sync 1, %0;" ::"r"(blockDim.x - 64) : "memory");
}

// Eight E4M3 codes (two words, low byte first) -> eight bf16, exactly.
// Through f16 (one cvt per pair): an E4M3 value is zero or a normal f16 (its
// smallest, 2^-9, is above f16's smallest normal 2^-14) whose low 7 mantissa
// bits are zero, so its bf16 is the sign, the exponent re-biased by
// 127 - 15 = 112 and the top 7 mantissa bits; zero halves stay zero.  (The
// quantizer saturates, so no code is NaN.)
__device__ __forceinline__ uint32_t f16x2_to_bf16x2(uint32_t h) {
    const uint32_t em = h & 0x7fff7fffu;
    const uint32_t r = ((em >> 3) & 0x0fff0fffu) + 0x38003800u;
    return (r & __vcmpne2(em, 0u)) | (h & 0x80008000u);
}
__device__ __forceinline__ uint4 e4m3x8_to_bf16x8(uint32_t a, uint32_t b) {
    return make_uint4(f16x2_to_bf16x2(e4m3x2_to_f16x2(a & 0xffffu)), f16x2_to_bf16x2(e4m3x2_to_f16x2(a >> 16)),
                      f16x2_to_bf16x2(e4m3x2_to_f16x2(b & 0xffffu)), f16x2_to_bf16x2(e4m3x2_to_f16x2(b >> 16)));
}
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ void am_take2(float& bv, int& bi, float v, int i) {
    if (v > bv || (v == bv && i < bi && v > -INFINITY)) {  // as the reference's fold: never -inf or NaN
        bv = v;
        bi = i;
    }
}

}  // namespace

// Epilogue of 16 activation columns of one weight row (packed row p of the
// matrix, TMEM lane `lr` of the super-tile): columns cb*16 .. +16 of the
// CTA's N-tile, activation rows m = n0 + cb*16 .. +16 of the launch.
template <int EPI>
__device__ __forceinline__ void tc_epilogue16(const GemmArgs& g, int p, int lr, int cb, int n0, float (&v)[16],
                                              float* am_v, int* am_i, int warp_e) {
    const GemvArgs& a = g.e;
    const int lane = lr & 31;
    const int tile = p >> 4, i16 = p & 15;
    // rows past the matrix (the last 16-row tile, the last 128-row CTA
    // tile) are computed but never stored
    const bool valid = tile < g.tiles16 && (EPI == EPI_SWIGLU || EPI == EPI_QKV || EPI == EPI_LOGITS || p < a.ldo);
    if (EPI != EPI_LOGITS && a.w8) {  // FP8 codes: the packed row's scale
        const float sc = valid ? a.wscale[p] : 0.f;
#pragma unroll
        for (int j = 0; j < 16; j++) v[j] *= sc;
    }
    // every global load of the 16 columns is issued before the arithmetic
    // that needs it (one round trip per group, not one per column)
    if (EPI == EPI_RESID) {
        uint16_t xo[16];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const int m = n0 + cb * 16 + j;
            xo[j] = (valid && m < a.M) ? __ldcg(a.out + (size_t)m * a.ldo + p) : (uint16_t)0;
        }
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const int m = n0 + cb * 16 + j;
            const bool live = valid && m < a.M;
            float sq = 0.f;
            if (live) {
                const float x = round_bf16(bf16_bits_to_f32(xo[j]) + round_bf16(v[j]));
                a.out[(size_t)m * a.ldo + p] = f32_to_bf16_bits(x);
                sq = x * x;
            }
            sq += __shfl_xor_sync(0xffffffffu, sq, 1);
            sq += __shfl_xor_sync(0xffffffffu, sq, 2);
            sq += __shfl_xor_sync(0xffffffffu, sq, 4);
            sq += __shfl_xor_sync(0xffffffffu, sq, 8);
            if (live && i16 == 0) a.ss_out[(size_t)m * kSsStride + tile] = sq;
        }
        return;
    }
    if (EPI == EPI_QKV) {
        const int hd = a.head_dim, half = hd >> 1, ppt = hd >> 4;
        const int q_dim = (a.q_tiles / ppt) * hd, kv_dim = a.n_kv * hd;
        const bool rope = tile < a.q_tiles + a.k_tiles, is_q = tile < a.q_tiles, first = i16 < 8;
        int h, d, d2, brow = 0, r = 0;
        if (rope) {
            const int t = is_q ? tile : tile - a.q_tiles;
            h = t / ppt;
            d = (t % ppt) * 8 + (i16 & 7);
            d2 = d + half;
            brow = is_q ? h * hd : q_dim + h * hd;
        } else {
            r = (tile - a.q_tiles - a.k_tiles) * kTileRows + i16;
            h = r / hd;
            d = d2 = r % hd;
        }
        const int dd = first ? d : d2;
        float b1 = 0.f, b2 = 0.f;
        if (a.bias && valid) {
            if (rope) {
                b1 = a.bias[brow + d];
                b2 = a.bias[brow + d2];
            } else {
                b1 = a.bias[q_dim + kv_dim + r];
            }
        }
        int pos[16], slot[16];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const int m = n0 + cb * 16 + j;
            const bool live = valid && m < a.M;
            pos[j] = live ? a.row_pos[m] : a.cap;
            slot[j] = live ? a.row_slot[m] : 0;
        }
        float cs[16], sn[16];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const bool ok = rope && pos[j] < a.cap;
            cs[j] = ok ? a.rope_cos[(size_t)pos[j] * hd + dd] : 0.f;
            sn[j] = ok ? a.rope_sin[(size_t)pos[j] * hd + dd] : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const int m = n0 + cb * 16 + j;
            const float partner = __shfl_xor_sync(0xffffffffu, v[j], 8);
            if (pos[j] >= a.cap) continue;  // also the rows past M and past the matrix
            if (rope) {
                const float x1 = (first ? v[j] : partner) + b1;
                const float x2 = (first ? partner : v[j]) + b2;
                const float y = first ? x1 * cs[j] - x2 * sn[j] : x2 * cs[j] + x1 * sn[j];
                if (is_q)
                    a.out[(size_t)m * a.ldo + h * hd + dd] = f32_to_bf16_bits(y);
                else
                    a.kcache[(((size_t)slot[j] * a.n_kv + h) * a.cap + pos[j]) * hd + dd] = f32_to_bf16_bits(y);
            } else {
                a.vcache[(((size_t)slot[j] * a.n_kv + h) * a.cap + pos[j]) * hd + d] = f32_to_bf16_bits(v[j] + b1);
            }
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < 16; j++) {
        const int m = n0 + cb * 16 + j;
        const bool live = valid && m < a.M;
        if (EPI == EPI_F32) {
            if (live) a.out_f32[(size_t)m * a.ldo + p] = v[j];
        } else if (EPI == EPI_SWIGLU) {
            const float partner = __shfl_xor_sync(0xffffffffu, v[j], 8);
            if (live && i16 < 8) {
                const float gt = v[j], up = partner;
                a.out[(size_t)m * a.ldo + tile * 8 + i16] = f32_to_bf16_bits(gt / (1.0f + expf(-gt)) * up);
            }
        } else if (EPI == EPI_LOGITS) {
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            const int pg = a.row0 + p;  // global vocabulary row
            if (live && pg < a.vocab) {
                const uint16_t b = f32_to_bf16_bits(v[j]);
                a.out[(size_t)m * a.ldo + pg] = b;
                const float f = bf16_bits_to_f32(b);
                if (f > -INFINITY) {  // the reference takes a value only if it beats -inf (NaN never)
                    bv = f;
                    bi = pg;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                am_take2(bv, bi, ov, oi);
            }
            if (lane == 0) {  // per-CTA slots of the N-tile's columns
                am_v[warp_e * kRowsCap + m - n0] = bv;
                am_i[warp_e * kRowsCap + m - n0] = bi;
            }
        }
    }
}

template <int EPI>
__global__ void __launch_bounds__(gemm_threads_max<EPI>(), 1) k_gemm_tc(const __grid_constant__ CUtensorMap tmap_x,
                                                             const __grid_constant__ CUtensorMap tmap_w, GemmArgs g) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const int kEpiW = (int)(blockDim.x - 64) >> 7;  // epilogue warps per lane quarter
    __shared__ __align__(8) unsigned long long full[kGemmMaxStages], empty[kGemmMaxStages], accum;
    __shared__ __align__(8) unsigned long long conv[kGemmMaxStages];  // FP8: a stage's A operand converted
    __shared__ uint32_t tmem_base_s;
    __shared__ int s_flag;
    __shared__ float am_v[EPI == EPI_LOGITS ? 4 * kRowsCap : 1];
    __shared__ int am_i[EPI == EPI_LOGITS ? 4 * kRowsCap : 1];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // CTA -> (super-tile S, N-tile nt, K split ksi); the N-tiles of a
    // super-tile are neighbours, so its weight tiles are read from HBM once
    // and from L2 by the others
    const int ksi = blockIdx.x % g.ks, t_sn = blockIdx.x / g.ks;
    const int S = t_sn / g.ntiles, n0 = (t_sn % g.ntiles) * g.N;
    const int kper = (g.kc + g.ks - 1) / g.ks;
    const int kb = min(g.kc, ksi * kper), ke = min(g.kc, kb + kper), nk = ke - kb;
    // each super-tile walks its k range from a different starting chunk, so
    // the CTAs in flight read different activation chunks (all CTAs read the
    // same x; in lock-step they would all hit the same L2 lines)
    // the split's chunks go in units of up to C consecutive chunks (one
    // weight copy and one activation copy each), walked from a per-super-
    // tile starting unit so that the CTAs in flight read different
    // activation chunks (all CTAs read the same x; in lock-step they would
    // all hit the same L2 lines)
    const int C = g.C, nu = (nk + C - 1) / C;
    const int rot = nu > 0 ? (int)(((unsigned)S * 2654435761u) % (unsigned)nu) : 0;
    const int N = g.N, SG = g.stages;
    // a stage: C bf16 weight tiles (the A operand), with FP8 weights then C
    // tiles of their codes (converted into the A tiles by the epilogue warps
    // during the mainloop), then C activation tiles
    const bool w8 = g.e.w8 != 0;
    const uint32_t stage_bytes = (uint32_t)C * (kStageA + (w8 ? kStageA8 : 0u) + (uint32_t)N * 128u);
    const uint32_t f8_off = (uint32_t)C * kStageA;
    const uint32_t b_off = (uint32_t)C * (kStageA + (w8 ? kStageA8 : 0u));
    const uint32_t bar_conv = (uint32_t)__cvta_generic_to_shared(&conv[0]);
    // 1024-byte alignment of the stage buffers (the swizzle atoms)
    const uint32_t smem0 = ((uint32_t)__cvta_generic_to_shared(smem_raw) + 1023u) & ~1023u;
    const uint32_t bar_full = (uint32_t)__cvta_generic_to_shared(&full[0]);
    const uint32_t bar_empty = (uint32_t)__cvta_generic_to_shared(&empty[0]);
    const uint32_t bar_acc = (uint32_t)__cvta_generic_to_shared(&accum);
    uint32_t ncols = 32;
    while ((int)ncols < N) ncols <<= 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SG; s++) {
            bar_init(bar_full + 8 * s, 1);
            bar_init(bar_empty + 8 * s, 1);
            bar_init(bar_conv + 8 * s, (blockDim.x - 64) / 32);  // one arrival per epilogue warp
        }
        bar_init(bar_acc, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        const uint32_t dst = (uint32_t)__cvta_generic_to_shared(&tmem_base_s);
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst), "r"(ncols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_s;
    bool failed = false;

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            // unit i: chunks c0 .. c0 + cnt - 1 of this split
            auto unit = [&](int i, int& c0, int& cnt) {
                const int u = (i + rot) % nu;
                c0 = kb + u * C;
                cnt = min(C, ke - c0);
            };
            auto issue_a = [&](int i) {
                int c0, cnt;
                unit(i, c0, cnt);
                // one copy of C chunks x 8 tiles (tiles past the matrix and
                // chunks past kc land as zeros); FP8 codes into the stage's
                // code tiles
                tensor_g2s_4d(smem0 + (uint32_t)(i % SG) * stage_bytes + (w8 ? f8_off : 0u), &tmap_w, 0, 0, 8 * S,
                              c0, bar_full + 8 * (i % SG));
            };
            const uint32_t tx_b = (uint32_t)N * 128u;
            auto issue_b = [&](int i) {
                int c0, cnt;
                unit(i, c0, cnt);
                const uint32_t dst = smem0 + (uint32_t)(i % SG) * stage_bytes + b_off;
                if (g.b3d) {
                    tensor_g2s_3d(dst, &tmap_x, 0, n0, c0, bar_full + 8 * (i % SG));
                } else {
                    for (int q = 0; q < cnt; q++)
                        tensor_g2s(dst + (uint32_t)q * tx_b, &tmap_x, (c0 + q) * kChunkK, n0, bar_full + 8 * (i % SG));
                }
            };
            auto tx_of = [&](int i) {
                int c0, cnt;
                unit(i, c0, cnt);
                return (uint32_t)C * (w8 ? kStageA8 : kStageA) + (uint32_t)(g.b3d ? C : cnt) * tx_b;
            };
            const int pre = min(SG, nu);
            // the weights do not depend on the previous kernel
            for (int i = 0; i < pre; i++) {
                bar_expect_tx(bar_full + 8 * (i % SG), tx_of(i));
                issue_a(i);
            }
            pdl_wait();
            for (int i = 0; i < pre; i++) issue_b(i);
            issued = pre;
            for (int i = pre; i < nu; i++) {
                const int s = i % SG;
                if (!bar_wait(bar_empty + 8 * s, (uint32_t)(((i / SG) - 1) & 1))) {
                    failed = true;
                    atomicExch(g.e.err, RENG_E_TIMEOUT);
                    break;
                }
                bar_expect_tx(bar_full + 8 * s, tx_of(i));
                issue_a(i);
                issue_b(i);
                issued = i + 1;
            }
            // drain: the last copy into each stage has landed before the CTA
            // may exit (already true unless a wait gave up; bounded)
            for (int i = max(0, issued - SG); i < issued; i++)
                if (!bar_wait(bar_full + 8 * (i % SG), (uint32_t)((i / SG) & 1)))
                    atomicExch(g.e.err, RENG_E_TIMEOUT);
        } else {
            pdl_wait();
        }
        pdl_launch();
    } else if (warp == 1) {
        pdl_wait();
        pdl_launch();
        if (lane == 0) {
            const uint32_t idesc = umma_idesc(N);
            int done = 0;
            for (int i = 0; i < nu; i++) {
                const int s = i % SG;
                if (!bar_wait(bar_full + 8 * s, (uint32_t)((i / SG) & 1)) ||
                    (w8 && !bar_wait(bar_conv + 8 * s, (uint32_t)((i / SG) & 1)))) {
                    atomicExch(g.e.err, RENG_E_TIMEOUT);
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const int cnt = min(C, ke - (kb + ((i + rot) % nu) * C));
                const uint32_t st0 = smem0 + (uint32_t)s * stage_bytes;
                for (int q = 0; q < cnt; q++) {
                    const uint32_t a0 = st0 + (uint32_t)q * kStageA, b0 = st0 + b_off + (uint32_t)q * (uint32_t)N * 128u;
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        umma(tmem, umma_desc(a0 + kk * 32), umma_desc(b0 + kk * 32), idesc,
                             (i > 0 || q > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(bar_empty + 8 * s);
                done = i + 1;
            }
            // the commit fires when every MMA issued so far has finished
            // (also after a wait gave up, so none still reads shared memory)
            if (done > 0) umma_commit(bar_acc);
            else bar_arrive(bar_acc);
        }
    } else {
        // ---- epilogue warps 2 .. 2 + 4 kEpiW ----
        pdl_wait();
        pdl_launch();
        const int q4 = warp & 3, warp_e = (warp - 2) & 3, eh = (warp - 2) >> 2;
        const int lr = 32 * q4 + lane;       // TMEM lane = row of the super-tile
        const int p = 128 * S + lr;          // packed row of the matrix
        if (w8) {
            // FP8 weights: while the MMAs run, every stage's codes become its
            // bf16 A tiles.  Epilogue thread ct converts 16-code pieces ct,
            // ct + nconv, ...: chunk q, row R of the super-tile, k 16 kq .. +16
            // (row R of a 2 KB-block pair at R * 128 bytes, 16-byte chunk j
            // at j ^ (R % 8), as the bf16 weight copies land).
            const int nconv = blockDim.x - 64, ct = threadIdx.x - 64;
            for (int i = 0; i < nu; i++) {
                const int s = i % SG;
                if (!failed && !bar_wait(bar_full + 8 * s, (uint32_t)((i / SG) & 1))) {
                    failed = true;
                    if (lane == 0) atomicExch(g.e.err, RENG_E_TIMEOUT);
                }
                if (!failed) {
                    const uint32_t st0 = smem0 + (uint32_t)s * stage_bytes;
                    for (int pc = ct; pc < C * 512; pc += nconv) {
                        const int q = pc >> 9, R = (pc >> 2) & 127, kq = pc & 3;
                        const uint4 f = lds128(st0 + f8_off + (uint32_t)q * kStageA8 + (uint32_t)R * 64u +
                                               (uint32_t)kq * 16u);
                        const uint32_t row = st0 + (uint32_t)q * kStageA + (uint32_t)R * 128u;
                        sts128(row + (uint32_t)(((2 * kq) ^ (R & 7)) << 4), e4m3x8_to_bf16x8(f.x, f.y));
                        sts128(row + (uint32_t)(((2 * kq + 1) ^ (R & 7)) << 4), e4m3x8_to_bf16x8(f.z, f.w));
                    }
                }
                // the A tiles are read by the tensor cores (async proxy)
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) bar_arrive(bar_conv + 8 * s);
            }
        }
        if (!bar_wait(bar_acc, 0)) {
            failed = true;
            if (lane == 0) atomicExch(g.e.err, RENG_E_TIMEOUT);
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t trow = tmem + ((uint32_t)(32 * q4) << 16);
        // no MMA ran (empty split, or a wait gave up and *err is set): the
        // accumulator was never written
        const bool zero = nk == 0 || failed;
        if (g.ks == 1) {
            for (int cb = eh; cb < N / 16; cb += kEpiW) {
                float v[16];
                tmem_ld16(trow + cb * 16, v);
                if (zero)
#pragma unroll
                    for (int j = 0; j < 16; j++) v[j] = 0.f;
                tc_epilogue16<EPI>(g, p, lr, cb, n0, v, am_v, am_i, warp_e);
            }
        } else if (g.gpart != nullptr) {
            // split K without a cluster: this split's partial to global
            // scratch [super-tile][split][128][N]; the last split of the
            // super-tile to arrive adds all of them in split order
            // (deterministic) and runs the epilogue
            float* mine = g.gpart + (((size_t)t_sn * g.ks + ksi) * 128 + lr) * N;
            for (int cb = eh; cb < N / 16; cb += kEpiW) {
                float v[16];
                tmem_ld16(trow + cb * 16, v);
#pragma unroll
                for (int j = 0; j < 4; j++)
                    __stcg(reinterpret_cast<float4*>(mine + cb * 16) + j,
                           zero ? make_float4(0.f, 0.f, 0.f, 0.f)
                                : make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
            }
            __threadfence();
            named_sync_epilogue();
            if (threadIdx.x == 64) s_flag = atomicAdd(g.gcnt + t_sn, 1) == g.ks - 1;
            named_sync_epilogue();
            if (s_flag) {
                __threadfence();
                for (int cb = eh; cb < N / 16; cb += kEpiW) {
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 16; j++) v[j] = 0.f;
                    for (int k = 0; k < g.ks; k++) {
                        const float4* src =
                            reinterpret_cast<const float4*>(g.gpart + (((size_t)t_sn * g.ks + k) * 128 + lr) * N + cb * 16);
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            const float4 x = __ldcg(src + j);
                            v[4 * j] += x.x;
                            v[4 * j + 1] += x.y;
                            v[4 * j + 2] += x.z;
                            v[4 * j + 3] += x.w;
                        }
                    }
                    tc_epilogue16<EPI>(g, p, lr, cb, n0, v, am_v, am_i, warp_e);
                }
                if (threadIdx.x == 64) g.gcnt[t_sn] = 0;
            }
        } else {
            // split K: this split's partial into the (finished) stage buffers,
            // row lr at lr * (N + 4) floats (conflict-free 16-byte stores)
            float* part = reinterpret_cast<float*>(smem_raw + (smem0 - (uint32_t)__cvta_generic_to_shared(smem_raw)));
            for (int cb = eh; cb < N / 16; cb += kEpiW) {
                float v[16];
                tmem_ld16(trow + cb * 16, v);
                float4* dst = reinterpret_cast<float4*>(part + (size_t)lr * (N + 4) + cb * 16);
#pragma unroll
                for (int j = 0; j < 4; j++)
                    dst[j] = zero ? make_float4(0.f, 0.f, 0.f, 0.f)
                                  : make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            }
        }
        if (EPI == EPI_LOGITS) {
            // CTA partials of every row: best over the 4 lane quarters
            named_sync_epilogue();
            const GemvArgs& a = g.e;
            // this CTA's best per row of its N-tile into the rows' running maxima
            for (int ml = threadIdx.x - 64; ml < min(N, a.M - n0); ml += 128 * kEpiW) {
                float bv = -INFINITY;
                int bi = 0x7fffffff;
                for (int w = 0; w < 4; w++) am_take2(bv, bi, am_v[w * kRowsCap + ml], am_i[w * kRowsCap + ml]);
                atomicMax(a.am_key + n0 + ml, am_pack(bv, bi));
            }
            __threadfence();
            named_sync_epilogue();
            if (threadIdx.x == 64) s_flag = (atomicAdd(a.am_count, 1u) == gridDim.x - 1);
            named_sync_epilogue();
            if (s_flag) {
                __threadfence();
                for (int m = threadIdx.x - 64; m < a.M; m += 128 * kEpiW) {
                    unsigned long long k = atomicExch(a.am_key + m, 0ull);
                    if (a.hx) k = head_exchange(a.hx, m, k, a.err);  // vocabulary shards of the ranks
                    am_i[m] = am_unpack(k);
                }
                named_sync_epilogue();
                if (a.hx && threadIdx.x == 64) *a.hx->epoch += 1;
                if (threadIdx.x == 64) {
                    if (a.mode == 0) {
                        const int s = *a.step;
                        for (int m = 0; m < a.M; m++) {
                            a.ids_ring[(size_t)(s + 1) * a.batch + m] = (uint32_t)am_i[m];
                            a.pos[m] += 1;
                        }
                        *a.step = s + 1;
                    } else {
                        *a.next_id = (uint32_t)am_i[a.M - 1];
                    }
                    *a.am_count = 0u;
                    __threadfence();
                }
            }
        }
    }
    if (g.ks > 1 && g.gpart == nullptr) {
        // the K splits of this super-tile are one cluster: once every
        // split's partial is in its shared memory, CTA r adds column blocks
        // r, r + ks, ... over the cluster in rank order (deterministic) and
        // runs their epilogue
        namespace cg = cooperative_groups;
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();
        if (warp >= 2) {
            const int lr = 32 * (warp & 3) + lane, p = 128 * S + lr, warp_e = (warp - 2) & 3, eh = (warp - 2) >> 2;
            float* part = reinterpret_cast<float*>(smem_raw + (smem0 - (uint32_t)__cvta_generic_to_shared(smem_raw)));
            for (int cb = ksi + eh * g.ks; cb < N / 16; cb += g.ks * kEpiW) {
                float v[16];
#pragma unroll
                for (int j = 0; j < 16; j++) v[j] = 0.f;
                for (int k = 0; k < g.ks; k++) {
                    const float4* src =
                        reinterpret_cast<const float4*>(cluster.map_shared_rank(part, k) + (size_t)lr * (N + 4) + cb * 16);
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const float4 x = src[j];
                        v[4 * j] += x.x;
                        v[4 * j + 1] += x.y;
                        v[4 * j + 2] += x.z;
                        v[4 * j + 3] += x.w;
                    }
                }
                tc_epilogue16<EPI>(g, p, lr, cb, n0, v, am_v, am_i, warp_e);
            }
        }
        cluster.sync();  // peers are done reading this CTA's partial
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
    }
}

// ------------------------------------------------------------ host side --
namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    });
    return fn;
}
}  // namespace

// Tensor map of a row-major bf16 activation buffer [rows][K] read in
// {64 k, n rows} boxes with 128-byte swizzle.
int gemm_tensor_map(const uint16_t* x, int rows, int K, int n, CUtensorMap* out) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(RENG_E_CUDA, "cuTensorMapEncodeTiled is not available");
    if (K % 8 || n % 16 || n < 16 || n > kRowsCap || n > rows || ((uintptr_t)x & 15))
        return fail(RENG_E_INVAL, "gemm_tensor_map: bad shape");
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)n};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void*)x, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(RENG_E_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return RENG_OK;
}

// Activations as {64 k, n rows, c chunks} boxes (128-byte swizzle): one copy
// fetches the x tiles of c consecutive 64-k chunks.  K must be a multiple of
// 64 (the chunk dimension would otherwise run into the next row).
int gemm_tensor_map3(const uint16_t* x, int rows, int K, int n, int c, CUtensorMap* out) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(RENG_E_CUDA, "cuTensorMapEncodeTiled is not available");
    if (K % kChunkK || n % 16 || n < 16 || n > kRowsCap || n > rows || c < 1 || c > 4 || ((uintptr_t)x & 15))
        return fail(RENG_E_INVAL, "gemm_tensor_map3: bad shape");
    cuuint64_t dims[3] = {(cuuint64_t)kChunkK, (cuuint64_t)rows, (cuuint64_t)(K / kChunkK)};
    cuuint64_t strides[2] = {(cuuint64_t)K * 2, (cuuint64_t)kChunkK * 2};
    cuuint32_t box[3] = {(cuuint32_t)kChunkK, (cuuint32_t)n, (cuuint32_t)c};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, (void*)x, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(RENG_E_CUDA, "cuTensorMapEncodeTiled (x, 3-D) failed (" + std::to_string((int)r) + ")");
    return RENG_OK;
}

// The packed weights [tiles16][kc][2 KB block] as a 4-D tensor {64 elements,
// 16 rows, tiles16, kc} read in {64, 16, 8, c} boxes: one copy lands c
// chunks of a 128-row super-tile as [c][8 tiles][2 KB], each chunk the
// UMMA A operand as packed (the blocks are stored pre-swizzled, so the copy
// itself does not swizzle).  Tiles past the matrix and chunks past kc read
// as zeros.
int gemm_weight_map(const uint8_t* w, int tiles16, int kc, int c, CUtensorMap* out) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(RENG_E_CUDA, "cuTensorMapEncodeTiled is not available");
    if (tiles16 < 1 || kc < 1 || c < 1 || c > 4 || ((uintptr_t)w & 15))
        return fail(RENG_E_INVAL, "gemm_weight_map: bad shape");
    cuuint64_t dims[4] = {64, (cuuint64_t)kTileRows, (cuuint64_t)tiles16, (cuuint64_t)kc};
    cuuint64_t strides[3] = {128, (cuuint64_t)kc * kBlockBytesBf16, (cuuint64_t)kBlockBytesBf16};
    cuuint32_t box[4] = {64, (cuuint32_t)kTileRows, 8, (cuuint32_t)c};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, (void*)w, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(RENG_E_CUDA, "cuTensorMapEncodeTiled (weights) failed (" + std::to_string((int)r) + ")");
    return RENG_OK;
}

int gemm_weight_map8(const uint8_t* w, int tiles16, int kc, int c, CUtensorMap* out) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(RENG_E_CUDA, "cuTensorMapEncodeTiled is not available");
    if (tiles16 < 1 || kc < 1 || c < 1 || c > 4 || ((uintptr_t)w & 15))
        return fail(RENG_E_INVAL, "gemm_weight_map8: bad shape");
    cuuint64_t dims[4] = {64, (cuuint64_t)kTileRows, (cuuint64_t)tiles16, (cuuint64_t)kc};
    cuuint64_t strides[3] = {64, (cuuint64_t)kc * kBlockBytesFp8, (cuuint64_t)kBlockBytesFp8};
    cuuint32_t box[4] = {64, (cuuint32_t)kTileRows, 8, (cuuint32_t)c};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, (void*)w, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(RENG_E_CUDA, "cuTensorMapEncodeTiled (FP8 weights) failed (" + std::to_string((int)r) + ")");
    return RENG_OK;
}

// A layer's K or V cache [slot][kv head][cap][hd] bf16 as 2-D rows of hd
// elements, read in {64, box_rows} boxes with the 128-byte swizzle (with 128
// rows, the tcgen05 operand layout of 128 keys x 64 head dims).  Rows past
// the last slot read as zeros.
int attn_cache_map(const uint16_t* cache, int hd, long long rows, int box_rows, CUtensorMap* out) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(RENG_E_CUDA, "cuTensorMapEncodeTiled is not available");
    if (hd % 64 || rows < 1 || box_rows < 8 || box_rows > 256 || box_rows % 8 || ((uintptr_t)cache & 15))
        return fail(RENG_E_INVAL, "attn_cache_map: bad shape");
    cuuint64_t dims[2] = {(cuuint64_t)hd, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)hd * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void*)cache, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(RENG_E_CUDA, "cuTensorMapEncodeTiled (cache) failed (" + std::to_string((int)r) + ")");
    return RENG_OK;
}

size_t gemm_smem_bytes(int n, int stages, int c, bool w8) {
    return (size_t)stages * c * (kStageA + (w8 ? kStageA8 : 0) + (size_t)n * 128) + 1024;
}

int gemm_chunks_per_stage(int n) {
    static const int fixed = [] {  // RENG_GEMM_C: chunks per stage, 1 or 2 (a tuning knob)
        const char* v = getenv("RENG_GEMM_C");
        const int x = v ? atoi(v) : 0;
        return x == 1 || x == 2 ? x : 0;
    }();
    return fixed ? fixed : 2;
    (void)n;
}

int gemm_pick_stages(int n, bool one_per_sm, int epi, int c, bool w8) {
    // Two CTAs per SM (no cluster): as many stages as fit in half the SM's
    // 228 KB beside the kernel's static shared memory, the 1 KB alignment
    // slack and the 1 KB per-CTA reservation (6 at N = 16, 5 at N = 32, 4 at
    // N = 64; one fewer for the LM head's argmax scratch).  One CTA per SM:
    // 4 stages; measured on B200 (Llama-8B widths, 64 rows), 8 stages at one
    // CTA per SM were slower than 4 (q/k/v 55 against 33 us).
    // stages of c chunks: the same bytes in flight as c x as many one-chunk stages
    const unsigned stage = (unsigned)c * (kStageA + (w8 ? kStageA8 : 0u) + (unsigned)n * 128u);
    const unsigned fixed = 2048u + (epi == EPI_LOGITS ? 9216u : 1024u);
    static const int one_sm = [] {  // RENG_GEMM_STAGES1: stages at one CTA per SM (a tuning knob)
        const char* v = getenv("RENG_GEMM_STAGES1");
        const int x = v ? atoi(v) : 0;
        return x >= 2 && x <= kGemmMaxStages ? x : 4;
    }();
    int s = one_per_sm ? (one_sm + c - 1) / c : (int)((114u * 1024u - fixed) / stage);
    const int fit = (int)((unsigned)kGemmStageBudget / stage);
    if (s > fit) s = fit;
    return s < 2 ? 2 : (s > kGemmMaxStages ? kGemmMaxStages : s);
}

template <int EPI>
static cudaError_t launch_tc_t(const CUtensorMap& map, const CUtensorMap& wmap, const GemmArgs& g, bool pdl,
                               cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    cfg.gridDim = dim3(g.super_tiles * g.ntiles * g.ks);
    cfg.blockDim = dim3(64 + 128 * (g.N > 64 || (g.e.w8 && g.N >= 64) ? epi_warps_max<EPI>() : 1));
    cfg.dynamicSmemBytes = gemm_smem_bytes(g.N, g.stages, g.C, g.e.w8 != 0);
    cfg.stream = st;
    int na = 0;
    if (g.ks > 1 && g.gpart == nullptr) {  // the K splits of a super-tile form one cluster
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = g.ks;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        na++;
    }
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, k_gemm_tc<EPI>, map, wmap, g);
}

// The largest dynamic shared memory any launch uses, and the whole of the
// SM's unified L1/shared storage as shared memory, so that two ~100 KB CTAs
// (N <= 64) fit on one SM (the default carveout sizes the SM for one block).
template <int EPI>
static cudaError_t prepare_t() {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_tc<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kGemmMaxDynSmem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_gemm_tc<EPI>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared);
    return e;
}

cudaError_t gemm_prepare() {
    cudaError_t e = prepare_t<EPI_QKV>();
    if (e == cudaSuccess) e = prepare_t<EPI_RESID>();
    if (e == cudaSuccess) e = prepare_t<EPI_SWIGLU>();
    if (e == cudaSuccess) e = prepare_t<EPI_LOGITS>();
    if (e == cudaSuccess) e = prepare_t<EPI_F32>();
    return e;
}

void gemm_plan(int super_tiles, int kc, int n, int epi, int sms, bool gsplit_ok, int* ks_out, int* stages_out,
               bool* gsplit_out, int* c_out, bool w8) {
    // Enough super-tiles to occupy the SMs (or the LM head, whose argmax
    // needs whole rows per CTA): one CTA per super-tile, two per SM at N <= 64.
    // Else split K over up to 8 CTAs.  At N = 16 the splits are plain CTAs
    // adding their partials through global scratch, two per SM with 6-stage
    // pipelines; wider, they form a cluster adding over shared memory
    // (clusters of these kernels are scheduled one CTA per SM).  Measured on
    // B200 (Llama-8B): down_proj at 8 rows 47 -> 30 us with plain splits (a
    // cluster of 4 per super-tile, 128 CTAs of 4 stages, kept about 72 KB in
    // flight per SM); at 64 rows plain splits lost (the last split reading
    // 8 partials of 32 KB: b64 step 6.98 -> 9.55 ms).
    int ks = 1;
    const bool gsplit = gsplit_ok && n <= 16;
    const int slots = gsplit ? 2 * sms : sms;
    if (epi != EPI_LOGITS && super_tiles < sms) {
        ks = slots / super_tiles;
        ks = ks < 1 ? 1 : (ks > kc ? kc : ks);
        if (ks > kGemmMaxSplits) ks = kGemmMaxSplits;
        const int kper = (kc + ks - 1) / ks;
        ks = (kc + kper - 1) / kper;  // every split gets at least one chunk
    }
    *ks_out = ks;
    *gsplit_out = ks > 1 && gsplit;
    // FP8 weights also stage their codes (one chunk per stage above 128
    // columns); from 64 columns they convert them with every epilogue warp,
    // one CTA per SM (measured on B200, Llama-8B FP8: b64 5776 -> 6215 tok/s;
    // at b16 two CTAs per SM with one warp per lane quarter stayed ahead,
    // 2049 against 1726)
    *c_out = w8 && n > 128 ? 1 : gemm_chunks_per_stage(n);
    *stages_out = gemm_pick_stages(n, (ks > 1 && !gsplit) || n > 64 || (w8 && n >= 64), epi, *c_out, w8);
}

cudaError_t launch_gemm_tc(const CUtensorMap& map, const CUtensorMap& wmap, const GemmArgs& g, int epi, bool pdl,
                           cudaStream_t st) {
    if (g.N % 16 || g.N < 16 || g.N > kRowsCap || g.ntiles < 1 || (g.ntiles > 1 && g.N != kRowsCap) ||
        g.e.M > g.N * g.ntiles || g.e.M > kGemmRowsMax || g.e.M < 1 || g.ks < 1 ||
        g.ks > kGemmMaxSplits || (epi == EPI_LOGITS && g.ks != 1) || g.stages < 2 || g.stages > kGemmMaxStages ||
        g.C < 1 || g.C > 4 || (g.b3d && g.kc * kChunkK != g.e.K) ||
        gemm_smem_bytes(g.N, g.stages, g.C, g.e.w8 != 0) > (size_t)kGemmMaxDynSmem || (g.e.w8 && !g.e.wscale) ||
        (g.ks > 1 && g.gpart == nullptr &&
         (size_t)g.stages * g.C * (kStageA + (size_t)g.N * 128) < (size_t)128 * (g.N + 4) * 4) ||
        (g.gpart != nullptr && g.gcnt == nullptr))
        return cudaErrorInvalidValue;
    switch (epi) {
        case EPI_QKV: return launch_tc_t<EPI_QKV>(map, wmap, g, pdl, st);
        case EPI_RESID: return launch_tc_t<EPI_RESID>(map, wmap, g, pdl, st);
        case EPI_SWIGLU: return launch_tc_t<EPI_SWIGLU>(map, wmap, g, pdl, st);
        case EPI_LOGITS: return launch_tc_t<EPI_LOGITS>(map, wmap, g, pdl, st);
        case EPI_F32: return launch_tc_t<EPI_F32>(map, wmap, g, pdl, st);
        default: return cudaErrorInvalidValue;
    }
}

// RMS-normalise M rows into a bf16 buffer (the x operand of the tcgen05
// GEMMs): xn = bf16(x * 1/sqrt(sum_t ss[m][t] / H + eps) * gain).
__global__ void __launch_bounds__(256) k_rmsnorm_rows(const uint16_t* x, const float* ss, int ss_tiles,
                                                      const float* gain, float eps, int H, uint16_t* xn) {
    const int m = blockIdx.x;
    __shared__ float inv_s;
    pdl_wait();
    pdl_launch();
    if (threadIdx.x < 32) {
        float s = 0.f;
        const float4* sp = reinterpret_cast<const float4*>(ss + (size_t)m * kSsStride);
        for (int t = threadIdx.x; t < ss_tiles / 4; t += 32) {
            const float4 v = sp[t];
            s += (v.x + v.y) + (v.z + v.w);
        }
        for (int t = (ss_tiles & ~3) + threadIdx.x; t < ss_tiles; t += 32) s += ss[(size_t)m * kSsStride + t];
        s = warp_sum(s);
        if (threadIdx.x == 0) inv_s = 1.0f / sqrtf(s / (float)H + eps);
    }
    __syncthreads();
    const float inv = inv_s;
    for (int k = threadIdx.x * 8; k < H; k += blockDim.x * 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(x + (size_t)m * H + k);
        const float4 g0 = *reinterpret_cast<const float4*>(gain + k);
        const float4 g1 = *reinterpret_cast<const float4*>(gain + k + 4);
        uint4 o;
        o.x = pack_bf16x2(bf16lo(v.x) * inv * g0.x, bf16hi(v.x) * inv * g0.y);
        o.y = pack_bf16x2(bf16lo(v.y) * inv * g0.z, bf16hi(v.y) * inv * g0.w);
        o.z = pack_bf16x2(bf16lo(v.z) * inv * g1.x, bf16hi(v.z) * inv * g1.y);
        o.w = pack_bf16x2(bf16lo(v.w) * inv * g1.z, bf16hi(v.w) * inv * g1.w);
        *reinterpret_cast<uint4*>(xn + (size_t)m * H + k) = o;
    }
}

cudaError_t launch_rmsnorm_rows(const uint16_t* x, const float* ss, int ss_tiles, const float* gain, float eps, int H,
                                uint16_t* xn, int M, bool pdl, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(M);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_rmsnorm_rows, x, ss, ss_tiles, gain, eps, H, xn);
}


// ------------------------------------------------------ reng_gemm_bf16 --
namespace {
struct DevFree {
    std::vector<void*> p;
    ~DevFree() {
        for (void* q : p) cudaFree(q);
    }
    template <typename T>
    cudaError_t alloc(T** out, size_t bytes) {
        cudaError_t e = cudaMalloc((void**)out, bytes < 16 ? 16 : bytes);
        if (e == cudaSuccess) p.push_back(*out);
        return e;
    }
};
}  // namespace

}  // namespace reng

#define GEMM_CU(x)                                                                        \
    do {                                                                                  \
        cudaError_t e__ = (x);                                                            \
        if (e__ != cudaSuccess)                                                           \
            return reng::fail(RENG_E_CUDA, std::string(#x) + ": " + cudaGetErrorString(e__)); \
    } while (0)

extern "C" int reng_gemm_bf16(const uint16_t* w, int rows, int K, const uint16_t* x, int M, float* y, int splits,
                              int iters, float* ms_out, int mem) {
    using namespace reng;
    RENG_CHECK_ARG(w && x && y, "reng_gemm_bf16: NULL buffer");
    RENG_CHECK_ARG(rows >= 1 && K >= 8 && K % 8 == 0, "reng_gemm_bf16: rows >= 1 and K a positive multiple of 8");
    RENG_CHECK_ARG(M >= 1 && M <= kGemmRowsMax, "reng_gemm_bf16: M must be in [1, 1024]");
    RENG_CHECK_ARG(splits >= -kGemmMaxSplits && splits <= kGemmMaxSplits && iters >= 0 && (iters == 0 || ms_out),
                   "reng_gemm_bf16: bad splits / iters");
    RENG_CHECK_ARG(mem == RENG_MEM_HOST || mem == RENG_MEM_DEVICE, "reng_gemm_bf16: bad mem");
    const cudaMemcpyKind h2d = mem == RENG_MEM_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
    const cudaMemcpyKind d2h = mem == RENG_MEM_HOST ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
    int dev = 0;
    GEMM_CU(cudaGetDevice(&dev));
    GEMM_CU(gemm_prepare());
    const int tiles = (rows + kTileRows - 1) / kTileRows, kc = (K + kChunkK - 1) / kChunkK;
    const int N = M > kRowsCap ? kRowsCap : (M + 15) / 16 * 16;  // N-tiles of kRowsCap beyond
    DevFree f;
    uint16_t *wd = nullptr, *xd = nullptr;
    uint8_t* packed = nullptr;
    int* rowmap = nullptr;
    float* yd = nullptr;
    int* err = nullptr;
    GEMM_CU(f.alloc(&wd, (size_t)rows * K * 2));
    GEMM_CU(f.alloc(&xd, (size_t)kGemmRowsMax * K * 2));
    GEMM_CU(f.alloc(&packed, (size_t)tiles * kc * kBlockBytesBf16));
    GEMM_CU(f.alloc(&rowmap, (size_t)tiles * kTileRows * 4));
    GEMM_CU(f.alloc(&yd, (size_t)M * rows * 4));
    GEMM_CU(f.alloc(&err, 4));
    GEMM_CU(cudaMemcpy(wd, w, (size_t)rows * K * 2, h2d));
    GEMM_CU(cudaMemset(xd, 0, (size_t)kGemmRowsMax * K * 2));
    GEMM_CU(cudaMemcpy(xd, x, (size_t)M * K * 2, h2d));
    GEMM_CU(cudaMemset(err, 0, 4));
    std::vector<int> map((size_t)tiles * kTileRows, -1);
    for (int r = 0; r < rows; r++) map[r] = r;
    GEMM_CU(cudaMemcpy(rowmap, map.data(), map.size() * 4, cudaMemcpyHostToDevice));
    PackArgs pa{};
    pa.src = wd;
    pa.ld = K;
    pa.rowmap = rowmap;
    pa.tiles = tiles;
    pa.K = K;
    pa.kc = kc;
    pa.dst = packed;
    GEMM_CU(launch_pack(pa, 0));

    GemmArgs g{};
    g.e.M = M;
    g.e.K = K;
    g.e.kc = kc;
    g.e.tiles = tiles;
    g.e.out_f32 = yd;
    g.e.ldo = rows;
    g.e.err = err;
    g.w = packed;
    g.tiles16 = tiles;
    g.kc = kc;
    g.super_tiles = (tiles + 7) / 8;
    g.N = N;
    g.ntiles = (M + N - 1) / N;
    bool gsplit = false;
    gemm_plan(g.super_tiles * g.ntiles, kc, N, EPI_F32, num_sms(dev), true, &g.ks, &g.stages, &gsplit, &g.C);
    if (splits != 0) {  // > 0: a cluster of that many splits; < 0: plain CTAs
        int s = splits > 0 ? splits : -splits;
        s = s > kc ? kc : s;
        if (s > kGemmMaxSplits) s = kGemmMaxSplits;
        const int kper = (kc + s - 1) / s;
        g.ks = (kc + kper - 1) / kper;
        gsplit = splits < 0 && g.ks > 1;
        g.stages = gemm_pick_stages(N, (g.ks > 1 && !gsplit) || N > 64, EPI_F32, g.C, false);
    }
    if (gsplit) {
        GEMM_CU(f.alloc(&g.gpart, (size_t)g.super_tiles * g.ntiles * g.ks * 128 * N * 4));
        GEMM_CU(f.alloc(&g.gcnt, (size_t)g.super_tiles * g.ntiles * 4));
        GEMM_CU(cudaMemset(g.gcnt, 0, (size_t)g.super_tiles * g.ntiles * 4));
    }
    CUtensorMap tmap, wmap;
    g.b3d = K % kChunkK == 0;
    int rc = g.b3d ? gemm_tensor_map3(xd, kGemmRowsMax, K, N, g.C, &tmap)
                   : gemm_tensor_map(xd, kGemmRowsMax, K, N, &tmap);
    if (rc) return rc;
    rc = gemm_weight_map(packed, tiles, kc, g.C, &wmap);
    if (rc) return rc;
    GEMM_CU(launch_gemm_tc(tmap, wmap, g, EPI_F32, false, 0));
    GEMM_CU(cudaDeviceSynchronize());
    if (iters > 0) {
        EventSet evs;
        GEMM_CU(evs.create(2));
        cudaEvent_t e0 = evs.e[0], e1 = evs.e[1];
        GEMM_CU(cudaEventRecord(e0, 0));
        for (int i = 0; i < iters; i++) GEMM_CU(launch_gemm_tc(tmap, wmap, g, EPI_F32, false, 0));
        GEMM_CU(cudaEventRecord(e1, 0));
        GEMM_CU(cudaEventSynchronize(e1));
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e0, e1);
        *ms_out = ms / (float)iters;
    }
    int herr = 0;
    GEMM_CU(cudaMemcpy(&herr, err, 4, cudaMemcpyDeviceToHost));
    if (herr) return fail(herr, "reng_gemm_bf16: the kernel gave up on a bounded wait");
    GEMM_CU(cudaMemcpy(y, yd, (size_t)M * rows * 4, d2h));
    return RENG_OK;
}
