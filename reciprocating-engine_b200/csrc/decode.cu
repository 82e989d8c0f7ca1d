// Decode-step kernels for B200 (sm_100a): packed-weight GEMV with fused
// RMSNorm and epilogues, split-K flash-decode GQA attention, embedding
// gather, and weight packing.
//
// Reference op sequence (crates/reng-synapse/src/model.rs:1172-1944 and the
// head at :2535-2664): rms1 -> q,k,v (+bias) -> RoPE -> KV write -> GQA
// attention -> o_proj -> +res -> rms2 -> gate,up -> SiLU*up -> down -> +res;
// final rms -> LM head -> bf16 logits -> argmax.  Here that is five kernels
// per layer plus an embedding gather and the LM head:
//
//   embed      x_res = embed[id]; norm partials of x_res
//   gemv<QKV>  rms1 (from partials) fused into the x fragments; q/k/v rows
//              paired (d, d+hd/2) per tile so RoPE is lane-local; k and v
//              written straight into the KV cache, q to a buffer
//   attn       split-K flash decode over the cache, last CTA combines
//   gemv<RES>  o_proj, x_res += bf16(o) in bf16, norm partials of x_res
//   gemv<SWIGLU> rms2 fused; gate/up rows paired per tile, silu(g)*u
//   gemv<RES>  down_proj, x_res += bf16(d), norm partials
//   gemv<LOGITS> final rms fused; bf16 logits; argmax partials, the last
//              CTA picks the ids (first index of the max), advances the
//              positions and the step counter
#include <algorithm>
#include <cstdlib>

#include <cooperative_groups.h>

#include "gemv_core.cuh"

namespace reng {

// ------------------------------------------------------------------ GEMV --

// The device pieces (x fragments, block MMAs, tile epilogues, the TMA ring
// primitives) are in gemv_core.cuh.

// Weight ring bytes of one warp with ST stages.
template <int ST>
__host__ __device__ constexpr int gemv_ring_bytes() {
    return ST * kChunkBytes;
}

// Ring stages issued before the wait on the previous kernel; the others go
// out after the x copy.  Measured on B200 (Llama-8B b1 step): 2 of 4 is
// 3.28 ms against 3.35 with all 4 ahead (x then queues behind 192 KB of
// weights per SM) and 3.38 with none.
constexpr int kPreStages = 2;

template <int EPI, int NWARP, int ST, int W8>
__global__ void __launch_bounds__(NWARP * 32) k_gemv(GemvArgs a, int use_smem) {
    extern __shared__ __align__(128) uint8_t smem_dyn[];
    // the warps' tile reduction; before the first tile it holds the RMS
    // partials of the rows (bulk-copied with x): 4-warp CTAs up to 2 KB,
    // 8-warp CTAs up to kMaxRows x 256 partials
    constexpr int kRedF4 = NWARP * 32, kSsF4 = NWARP == 4 ? kRedF4 : kMaxRows * 256 / 4;
    __shared__ __align__(16) float4 red_buf[kRedF4 > kSsF4 ? kRedF4 : kSsF4];
    float4(*red)[32] = reinterpret_cast<float4(*)[32]>(red_buf);
    __shared__ float inv_s[kMaxRows];
    __shared__ int s_ids[kMaxRows];
    __shared__ int s_last;
    __shared__ __align__(8) unsigned long long bars[NWARP * ST];
    __shared__ __align__(8) unsigned long long xbar;
    const int K = a.K;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const int kc_per = (a.kc + NWARP - 1) / NWARP;
    const int c0 = min(a.kc, warp * kc_per), c1 = min(a.kc, c0 + kc_per);
    constexpr int BB = W8 ? kBlockBytesFp8 : kBlockBytesBf16;  // bytes per block
    constexpr int CB = kChunkBytes / BB;                        // blocks per chunk
    constexpr int NP = W8 ? 2 : 4;                              // 16-byte pieces per lane per block
    int poff[4];
    lane_pieces<W8>(g, q, lane, poff);
    const int nct = max(1, (c1 - c0 + CB - 1) / CB);
    const int ntile = blockIdx.x < a.tiles ? (a.tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int nchunks = ntile * nct;

    // chunk j -> its first block and block count (0 for an empty k-range)
    auto chunk_src = [&](int j, int& nb) -> const uint8_t* {
        const int tile = blockIdx.x + (j / nct) * gridDim.x;
        const int b0 = c0 + (j % nct) * CB;
        nb = max(0, min(CB, c1 - b0));
        return a.w + ((size_t)tile * a.kc + b0) * BB;
    };

    // ---- start the weight stream (independent of the previous kernel) ----
    const uint32_t ring = (uint32_t)__cvta_generic_to_shared(smem_dyn) + warp * gemv_ring_bytes<ST>();  // per warp
    const uint32_t bar0 = (uint32_t)__cvta_generic_to_shared(&bars[0]) + warp * ST * 8;
    bool failed = false;
    int issued = 0;  // lane 0: chunks whose copy was issued
    int waited = 0;  // chunks whose copy was waited for
    auto tma_issue = [&](int j) {  // lane 0 only
        if (j >= nchunks || failed) return;
        int nb;
        const uint8_t* src = chunk_src(j, nb);
        const uint32_t bar = bar0 + (j % ST) * 8;
        const uint32_t bytes = (uint32_t)nb * BB;
        mbar_expect_tx(bar, bytes);
        if (bytes) tma_load_1d(ring + (j % ST) * kChunkBytes, src, bytes, bar);
        issued = j + 1;
    };
    const uint32_t xbar_a = (uint32_t)__cvta_generic_to_shared(&xbar);
    if (threadIdx.x == 0 && use_smem) {
        mbar_init(xbar_a, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (lane == 0) {
        for (int s2 = 0; s2 < ST; s2++) mbar_init(bar0 + s2 * 8, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int j = 0; j < kPreStages; j++) tma_issue(j);
    }
    __syncwarp();
    // the RMSNorm gains of this thread's k-groups (constants: before the wait)
    constexpr int GV = NWARP == 4 ? 5 : 3;  // k-groups per thread: K <= 5120 (4 warps), 6144 (8)
    float4 gp[GV][2];
    const bool gain_pre = a.ss_in != nullptr && use_smem && K / 8 <= GV * NWARP * 32;
    if (gain_pre) gain_preload<GV>(a, K, gp);

    pdl_wait();
    pdl_launch();

    // x rows (written by the previous kernel): one bulk copy per row into
    // shared memory, while the warps reduce the RMS partials
    const int xstride = gemv_xstride(K);
    uint16_t* xsm = reinterpret_cast<uint16_t*>(smem_dyn + NWARP * gemv_ring_bytes<ST>());
    // the RMS partials ride with x when they fit the reduction buffer (plain
    // loads here queue behind the weight stream already in flight: 2-3 us)
    const bool ss_tma = a.ss_in != nullptr && use_smem && (a.ss_tiles & 3) == 0 &&
                        a.M * a.ss_tiles * 4 <= (int)sizeof(red_buf);
    if (use_smem) {
        __syncthreads();  // barrier init visible to every thread before any wait
        if (threadIdx.x == 0) {
            const uint32_t ssb = (uint32_t)(a.ss_tiles * 4);
            mbar_expect_tx(xbar_a, (uint32_t)(a.M * K * 2) + (ss_tma ? a.M * ssb : 0u));
            for (int m = 0; m < a.M; m++)
                tma_load_1d((uint32_t)__cvta_generic_to_shared(xsm + m * xstride), a.x + (size_t)m * a.ldx,
                            (uint32_t)(K * 2), xbar_a);
            if (ss_tma)
                for (int m = 0; m < a.M; m++)
                    tma_load_1d((uint32_t)__cvta_generic_to_shared(red_buf) + m * ssb, a.ss_in + (size_t)m * kSsStride,
                                ssb, xbar_a);
        }
    }
    // the rest of the ring behind x (the copies issued so far stand in front
    // of x in the SM's queue)
    __syncwarp();
    if (lane == 0)
        for (int j = kPreStages; j < ST; j++) tma_issue(j);
    __syncwarp();
    if (a.ss_in != nullptr && !ss_tma) {
        for (int m = warp; m < a.M; m += NWARP) {
            float s = 0.0f;
            const float4* sp = reinterpret_cast<const float4*>(a.ss_in + (size_t)m * kSsStride);
#pragma unroll 4
            for (int t = lane; t < a.ss_tiles / 4; t += 32) {
                const float4 v = sp[t];
                s += (v.x + v.y) + (v.z + v.w);
            }
            for (int t = (a.ss_tiles & ~3) + lane; t < a.ss_tiles; t += 32) s += a.ss_in[(size_t)m * kSsStride + t];
            s = warp_sum(s);
            if (lane == 0) inv_s[m] = 1.0f / sqrtf(s / (float)a.norm_k + a.eps);
        }
    }
    const uint16_t* xs = nullptr;
    if (use_smem) {
        if (!mbar_wait_bounded(xbar_a, 0)) {
            failed = true;
            if (threadIdx.x == 0) atomicExch(a.err, RENG_E_TIMEOUT);
        }
        if (ss_tma) {
            for (int m = warp; m < a.M; m += NWARP) {
                const float4* sp = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(red_buf) + m * a.ss_tiles);
                float s = 0.0f;
                for (int t = lane; t < a.ss_tiles / 4; t += 32) {
                    const float4 v = sp[t];
                    s += (v.x + v.y) + (v.z + v.w);
                }
                s = warp_sum(s);
                if (lane == 0) inv_s[m] = 1.0f / sqrtf(s / (float)a.norm_k + a.eps);
            }
        }
        __syncthreads();
        if (a.ss_in != nullptr) {
            if (gain_pre) normalise_x_pre<W8, GV>(a, xsm, xstride, K, inv_s, gp);
            else normalise_x<W8>(a, xsm, xstride, K, inv_s);
            __syncthreads();
        } else if (W8) {
            x_to_f16(a, xsm, xstride, K);
            __syncthreads();
        }
        xs = xsm;
    } else if (a.ss_in != nullptr) {
        __syncthreads();
    }

    float best_v[2] = {-INFINITY, -INFINITY};
    int best_i[2] = {0, 0};
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < nchunks; j++) {
        const int b0 = c0 + (j % nct) * CB;
        const uint32_t bar = bar0 + (j % ST) * 8;
        if (!failed) {
            if (mbar_wait_bounded(bar, (uint32_t)((j / ST) & 1))) {
                waited = j + 1;
            } else {
                failed = true;
                if (lane == 0) atomicExch(a.err, RENG_E_TIMEOUT);
            }
        }
        const uint32_t st = ring + (j % ST) * kChunkBytes;
#pragma unroll
        for (int b = 0; b < CB; b++)
            if (b0 + b < c1) {
                uint4 v[4];
#pragma unroll
                for (int p = 0; p < NP; p++) v[p] = lds128(st + b * BB + poff[p]);
                block_mma<W8>(acc, v, a, xs, xstride, K, b0 + b, g, q);
            }
        // the stage is read: let the async proxy refill it
        __syncwarp();
        if (lane == 0) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tma_issue(j + ST);
        }
        __syncwarp();
        if ((j % nct) != nct - 1) continue;
        // ---- a tile is complete: reduce the warps' k-slices on warp 0 ----
        const int tile = blockIdx.x + (j / nct) * gridDim.x;
        if (NWARP > 1) {
            __syncthreads();
            red[warp][lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
            __syncthreads();
            if (warp == 0) {
#pragma unroll
                for (int w = 1; w < NWARP; w++) {
                    float4 r = red[w][lane];
                    acc[0] += r.x;
                    acc[1] += r.y;
                    acc[2] += r.z;
                    acc[3] += r.w;
                }
            }
        }
        if (warp == 0) {
            if (W8) {  // per-row scale of the FP8 codes
                const float s0 = a.wscale[tile * kTileRows + g], s1 = a.wscale[tile * kTileRows + g + 8];
                acc[0] *= s0;
                acc[1] *= s0;
                acc[2] *= s1;
                acc[3] *= s1;
            }
            gemv_epilogue<EPI>(a, tile, acc, g, q, best_v, best_i);
        }
        acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
    }
    if (failed && lane == 0) {
        // drain this warp's own copies still in flight before exiting (bounded)
        for (int jj = waited; jj < issued; jj++)
            if (!mbar_wait_bounded(bar0 + (jj % ST) * 8, (uint32_t)((jj / ST) & 1))) break;
    }

    if (EPI == EPI_LOGITS) {
        // this CTA's best per row into the rows' running maxima (lanes g == 0
        // of warp 0 hold rows 2q, 2q + 1); the last CTA reads them out
        if (warp == 0 && g == 0) {
            if (2 * q < a.M) atomicMax(a.am_key + 2 * q, am_pack(best_v[0], best_i[0]));
            if (2 * q + 1 < a.M) atomicMax(a.am_key + 2 * q + 1, am_pack(best_v[1], best_i[1]));
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) s_last = (atomicAdd(a.am_count, 1u) == gridDim.x - 1);
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        if (threadIdx.x < a.M) {
            unsigned long long k = atomicExch(a.am_key + threadIdx.x, 0ull);
            if (a.hx) k = head_exchange(a.hx, threadIdx.x, k, a.err);  // vocabulary shards of the ranks
            s_ids[threadIdx.x] = am_unpack(k);
        }
        __syncthreads();
        if (a.hx && threadIdx.x == 0) *a.hx->epoch += 1;
        if (threadIdx.x == 0) {
            if (a.mode == 0) {
                const int s = *a.step;
                for (int m = 0; m < a.M; m++) {
                    a.ids_ring[(size_t)(s + 1) * a.batch + m] = (uint32_t)s_ids[m];
                    a.pos[m] += 1;
                }
                *a.step = s + 1;
            } else {
                *a.next_id = (uint32_t)s_ids[a.M - 1];
            }
            *a.am_count = 0u;
            __threadfence();
        }
    }
}

// Shared x copy of a launch with an nw-warp ring: staged when it fits beside
// the ring (normalised inputs always: they are normalised in place); else
// the fragments are read from global memory.
static size_t gemv_xbytes(const GemvArgs& a, int nw) {
    size_t b = (size_t)a.M * gemv_xstride(a.K) * 2;
    const bool need = a.ss_in != nullptr;
    if (need || (b <= kGemvMaxSmem && (size_t)nw * gemv_ring_bytes<kTmaStages>() + b <= 200 * 1024)) return b;
    return 0;
}

template <int EPI, int NW, int ST>
static cudaError_t prepare_st() {
    cudaError_t e = cudaFuncSetAttribute(k_gemv<EPI, NW, ST, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_gemv<EPI, NW, ST, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    return e;
}

// CTAs of k_gemv<EPI, NW, ST, W8> resident per SM with smem dynamic bytes.
template <int EPI, int NW, int ST, int W8>
static int gemv_per_sm(size_t smem) {
    int per_sm = 0;
    if (smem > 200 * 1024) return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_gemv<EPI, NW, ST, W8>, NW * 32, smem) != cudaSuccess)
        return 0;
    return per_sm;
}

template <int EPI, int NW, int ST, int W8>
static cudaError_t launch_one(const GemvArgs& a, int per_sm, int max_grid, bool pdl, cudaStream_t st,
                              int* grid_out) {
    const size_t xbytes = gemv_xbytes(a, NW);
    const size_t smem = (size_t)NW * gemv_ring_bytes<ST>() + xbytes;
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = num_sms(dev);
    int cap = sms * std::max(1, per_sm);
    if (max_grid > 0 && max_grid < cap) cap = max_grid;
    // persistent grid of every resident slot (tiles interleaved over the
    // CTAs), so each SM holds the same number of CTAs: the weight stream of
    // an SM is capped (about 50 GB/s measured on B200, two or three CTAs
    // alike), so equal tiles per SM, not per CTA, is the balance that counts
    // (gate/up at Llama-8B b1: 359 CTAs of 5 tiles left 63 SMs with 15
    // tiles against 10 on the rest, a 10 us tail).  The LM head keeps equal
    // tiles per CTA: measured 150 against 161 us with every slot filled.
    int grid = std::min(a.tiles, cap);
    if (EPI == EPI_LOGITS) {
        const int per = (a.tiles + cap - 1) / cap;
        grid = (a.tiles + per - 1) / per;
    }
    if (grid_out) *grid_out = grid;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(NW * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_gemv<EPI, NW, ST, W8>, a, xbytes > 0 ? 1 : 0);
}

// Ring depth: 4 stages of 4 KB per warp, three 4-warp CTAs per SM.  Deeper
// rings for the projections whose tiles fit one wave at two CTAs per SM
// (o_proj 6 stages, down_proj 5, Llama-8B b1) made those kernels faster
// alone but the step slower, 3.24 against 3.18 ms (their shared memory
// keeps the next kernel's CTAs from starting early).
template <int EPI, int NW, int W8>
static cudaError_t launch_stages(const GemvArgs& a, int max_grid, bool pdl, cudaStream_t st, int* grid_out) {
    const int p4 = gemv_per_sm<EPI, NW, 4, W8>((size_t)NW * gemv_ring_bytes<4>() + gemv_xbytes(a, NW));
    if (p4 < 1) return cudaErrorInvalidValue;
    return launch_one<EPI, NW, 4, W8>(a, p4, max_grid, pdl, st, grid_out);
}

template <int EPI>
static cudaError_t prepare_t() {
    cudaError_t e = prepare_st<EPI, 4, 4>();
    if (e == cudaSuccess) e = prepare_st<EPI, 8, 4>();
    return e;
}

// Allow the large dynamic shared memory of every GEMV instantiation on the
// current device (must run before a stream capture).
cudaError_t gemv_prepare() {
    cudaError_t e = prepare_t<EPI_QKV>();
    if (e == cudaSuccess) e = prepare_t<EPI_RESID>();
    if (e == cudaSuccess) e = prepare_t<EPI_SWIGLU>();
    if (e == cudaSuccess) e = prepare_t<EPI_LOGITS>();
    if (e == cudaSuccess) e = prepare_t<EPI_F32>();
    return e;
}

// shape = warps per CTA (4 or 8) + 100 (the TMA weight ring)
template <int EPI>
static cudaError_t launch_gemv_t(const GemvArgs& a, int shape, int max_grid, bool pdl, cudaStream_t st,
                                 int* grid_out) {
    switch (shape) {
        case 104: return a.w8 ? launch_stages<EPI, 4, 1>(a, max_grid, pdl, st, grid_out)
                              : launch_stages<EPI, 4, 0>(a, max_grid, pdl, st, grid_out);
        case 108: return a.w8 ? launch_stages<EPI, 8, 1>(a, max_grid, pdl, st, grid_out)
                              : launch_stages<EPI, 8, 0>(a, max_grid, pdl, st, grid_out);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemv(const GemvArgs& a, int epi, int shape, int max_grid, bool pdl, cudaStream_t st,
                        int* grid_out) {
    switch (epi) {
        case EPI_QKV: return launch_gemv_t<EPI_QKV>(a, shape, max_grid, pdl, st, grid_out);
        case EPI_RESID: return launch_gemv_t<EPI_RESID>(a, shape, max_grid, pdl, st, grid_out);
        case EPI_SWIGLU: return launch_gemv_t<EPI_SWIGLU>(a, shape, max_grid, pdl, st, grid_out);
        case EPI_LOGITS: return launch_gemv_t<EPI_LOGITS>(a, shape, max_grid, pdl, st, grid_out);
        case EPI_F32: return launch_gemv_t<EPI_F32>(a, shape, max_grid, pdl, st, grid_out);
        default: return cudaErrorInvalidValue;
    }
}

// ------------------------------------------------------------- attention --
// Decode attention over the KV cache.  One thread-block cluster of up to
// kAttnCluster CTAs per (row, KV group) (fewer when the rows x groups
// already fill the GPU, chosen at launch): CTA s takes the s-th contiguous
// slice of the row's keys 0..pos and runs an f32 online softmax over it in
// kAttnChunk-key shared-memory tiles, for all hpg query heads of the group at
// once (each K/V tile is read once for the whole GQA group).  The slices are
// then combined through distributed shared memory: after a cluster barrier
// every CTA reads the (max, sum, unnormalised output) of all slices for its
// share of the outputs and writes them as bf16.  No global scratch, no
// atomics, one launch; the cluster barriers are hardware barriers.
constexpr int kAttnThreads = 256;
constexpr int kAttnMaxHpg = 8;
constexpr int kAttnMaxHd = 128;

__global__ void __launch_bounds__(kAttnThreads) k_attn(AttnArgs a) {
    namespace cg = cooperative_groups;
    constexpr int CH = kAttnChunk;
    constexpr int KP = kAttnMaxHd + 8;  // padded row (bf16): conflict-free 16-byte reads
    __shared__ __align__(16) uint16_t Ks[CH * KP];
    __shared__ __align__(16) uint16_t Vs[CH * KP];
    __shared__ __align__(16) float Qs[kAttnMaxHpg * kAttnMaxHd];
    __shared__ float Ps[kAttnMaxHpg][CH];
    __shared__ float Ms[kAttnMaxHpg], Ls[kAttnMaxHpg], Al[kAttnMaxHpg];
    __shared__ __align__(16) float Os[kAttnMaxHpg * kAttnMaxHd];  // this slice's unnormalised output

    cg::cluster_group cluster = cg::this_cluster();
    const int s = (int)cluster.block_rank(), ns = (int)cluster.num_blocks();
    const int grp = blockIdx.y, m = blockIdx.z;
    const int hd = a.hd, hpg = a.hpg, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // Before the wait on the q/k/v kernel: the row's position and slot (set
    // by the step's embedding gather, two launches back) and this slice's
    // first key tile except the keys that kernel writes (the current
    // position; in a prefill block every position from the block's first).
    const int pos = __ldcg(a.row_pos + m);
    const int nkeys = min(pos + 1, a.cap);
    const int per = (nkeys + ns - 1) / ns;
    const int k0 = min(nkeys, s * per), k1 = min(nkeys, k0 + per);
    const int slot = __ldcg(a.row_slot + m);
    const size_t cache_base = (((size_t)slot * a.n_kv + grp) * a.cap) * hd;
    const int q_dim = a.n_kv * hpg * hd;
    const int vec_per_row = hd / 8;
    const int old_end = pos - (a.contiguous ? m : 0);  // keys below were written by earlier launches
    const int kn_first = min(CH, k1 - k0);
    const int pre_end = max(k0, min(k0 + kn_first, old_end));
    auto load_keys = [&](int c0, int j0, int j1) {  // keys [c0 + j0, c0 + j1) into tile rows j0..j1-1
        for (int i = j0 * vec_per_row + tid; i < j1 * vec_per_row; i += kAttnThreads) {
            const int j = i / vec_per_row, v = i % vec_per_row;
            const size_t off = cache_base + (size_t)(c0 + j) * hd + v * 8;
            *reinterpret_cast<uint4*>(&Ks[j * KP + v * 8]) = __ldcg(reinterpret_cast<const uint4*>(a.kcache + off));
            *reinterpret_cast<uint4*>(&Vs[j * KP + v * 8]) = __ldcg(reinterpret_cast<const uint4*>(a.vcache + off));
        }
    };
    if (k0 < k1) load_keys(k0, 0, pre_end - k0);
    pdl_wait();
    pdl_launch();

    const uint16_t* qrow = a.q + (size_t)m * q_dim + (size_t)grp * hpg * hd;
    for (int i = tid; i < hpg * hd; i += kAttnThreads) Qs[i] = bf16_bits_to_f32(qrow[i]);
    if (tid < kAttnMaxHpg) {
        Ms[tid] = -INFINITY;
        Ls[tid] = 0.f;
    }
    // PV ownership: thread -> (head, 4 output dims); hpg * hd / 4 <= 256
    const int per_head = hd / 4;
    const int ph = tid / per_head, pd = (tid % per_head) * 4;
    const bool owns = tid < hpg * per_head;
    float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;

    for (int c0 = k0; c0 < k1; c0 += CH) {
        const int kn = min(CH, k1 - c0);
        __syncthreads();  // previous tile fully consumed (and Qs/Ms ready on the first)
        load_keys(c0, c0 == k0 ? pre_end - k0 : 0, kn);
        __syncthreads();
        // scores: thread -> key j, heads h = t/CH, t/CH + 4, ...
        {
            const int j = tid % CH;
            for (int h = tid / CH; h < hpg; h += kAttnThreads / CH) {
                float sc = -INFINITY;
                if (j < kn) {
                    float acc = 0.f;
                    const float* qh = Qs + h * hd;
                    for (int d = 0; d < hd; d += 8) {
                        uint4 kv = *reinterpret_cast<const uint4*>(&Ks[j * KP + d]);
                        acc += qh[d + 0] * bf16lo(kv.x) + qh[d + 1] * bf16hi(kv.x) +
                               qh[d + 2] * bf16lo(kv.y) + qh[d + 3] * bf16hi(kv.y) +
                               qh[d + 4] * bf16lo(kv.z) + qh[d + 5] * bf16hi(kv.z) +
                               qh[d + 6] * bf16lo(kv.w) + qh[d + 7] * bf16hi(kv.w);
                    }
                    sc = acc;
                }
                Ps[h][j] = sc;
            }
        }
        __syncthreads();
        // online-softmax statistics: warp h
        if (warp < hpg) {
            const int h = warp;
            float mx = -INFINITY;
            for (int j = lane; j < CH; j += 32) mx = fmaxf(mx, Ps[h][j]);
            mx = warp_max(mx);
            const float m_old = Ms[h], m_new = fmaxf(m_old, mx);
            float sum = 0.f;
            for (int j = lane; j < CH; j += 32) {
                const float p = (j < kn) ? expf(Ps[h][j] - m_new) : 0.f;
                Ps[h][j] = p;
                sum += p;
            }
            sum = warp_sum(sum);
            if (lane == 0) {
                const float alpha = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
                Al[h] = alpha;
                Ls[h] = Ls[h] * alpha + sum;
                Ms[h] = m_new;
            }
        }
        __syncthreads();
        if (owns) {
            const float al = Al[ph];
            acc0 *= al;
            acc1 *= al;
            acc2 *= al;
            acc3 *= al;
            for (int j = 0; j < kn; j++) {
                const float p = Ps[ph][j];
                uint2 vv = *reinterpret_cast<const uint2*>(&Vs[j * KP + pd]);
                acc0 += p * bf16lo(vv.x);
                acc1 += p * bf16hi(vv.x);
                acc2 += p * bf16lo(vv.y);
                acc3 += p * bf16hi(vv.y);
            }
        }
    }
    if (owns) *reinterpret_cast<float4*>(&Os[ph * hd + pd]) = make_float4(acc0, acc1, acc2, acc3);
    cluster.sync();  // every slice's (Ms, Ls, Os) is complete and visible cluster-wide

    // combine: CTA s writes outputs o = s, s + ns, ... of the hpg * hd
    for (int o = s + ns * tid; o < hpg * hd; o += ns * kAttnThreads) {
        const int h = o / hd, d = o % hd;
        float mx = -INFINITY;
        for (int r = 0; r < ns; r++) mx = fmaxf(mx, *cluster.map_shared_rank(&Ms[h], r));
        float num = 0.f, den = 0.f;
        for (int r = 0; r < ns; r++) {
            const float mr = *cluster.map_shared_rank(&Ms[h], r);
            const float w = (mr == -INFINITY) ? 0.f : expf(mr - mx);
            num += w * *cluster.map_shared_rank(&Os[h * hd + d], r);
            den += w * *cluster.map_shared_rank(&Ls[h], r);
        }
        a.out[(size_t)m * q_dim + ((size_t)grp * hpg + h) * hd + d] = f32_to_bf16_bits(num / den);
    }
    cluster.sync();  // keep this CTA's shared memory alive until its peers have read it
}

// Key slices per (row, KV group): 8 (a cluster) when the rows x groups are
// few, fewer as they grow.  Measured on B200 (Llama-8B, 8 KV groups): b1 (8
// units) 8 slices; b8 (64 units) 4 beat 8 and 2 (7.9 against 10.0 and 9.2
// us); b16 4 beat 8 (10.6 against 19.2 us); b64 (512 units) 1 beat 2 and 4
// (24.9 against 27.9 and 39.5 us).
int attn_slices(long long units) {
    static const int fixed_ns = [] {  // RENG_ATTN_SLICES: a tuning knob fixing the slices (1, 2, 4 or 8)
        const char* v = getenv("RENG_ATTN_SLICES");
        const int x = v ? atoi(v) : 0;
        return x == 1 || x == 2 || x == 4 || x == 8 ? x : 0;
    }();
    if (fixed_ns) return fixed_ns;
    int dev = 0;
    cudaGetDevice(&dev);
    return units >= 2LL * num_sms(dev) ? 1 : units >= 64 ? 4 : kAttnCluster;
}

cudaError_t launch_attn(const AttnArgs& a, int /*chunk*/, bool pdl, cudaStream_t st) {
    if (a.hpg > kAttnMaxHpg || a.hd > kAttnMaxHd || a.hd % 8 || a.hpg * (a.hd / 4) > kAttnThreads)
        return cudaErrorInvalidValue;
    const int ns = attn_slices((long long)a.M * a.n_kv);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    cfg.gridDim = dim3(ns, a.n_kv, a.M);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = ns;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, k_attn, a);
}

// --------------------------------------------------------------- q/k norm --
// One warp per (head, row): RMS over the head, the gain, then rotate-half
// RoPE at the row's position (crates/reng-synapse/src/model.rs:2962-3010:
// head_norm before rope_head).  The head is staged in shared memory for the
// rotation's partner element.
__global__ void __launch_bounds__(32) k_qk_norm(QkNormArgs a) {
    __shared__ float t[kAttnMaxHd];
    const int j = blockIdx.x, m = blockIdx.y, lane = threadIdx.x;
    pdl_wait();
    pdl_launch();
    const int pos = __ldcg(a.row_pos + m);
    if (pos >= a.cap) return;  // as the q/k/v epilogue: such a row wrote nothing
    const int hd = a.hd, half = hd >> 1;
    uint16_t* p;
    const float* g;
    if (j < a.nq) {
        p = a.q + (size_t)m * a.q_dim + (size_t)j * hd;
        g = a.qn;
    } else {
        const int slot = __ldcg(a.row_slot + m);
        p = a.kcache + (((size_t)slot * a.n_kv + (j - a.nq)) * a.cap + pos) * hd;
        g = a.kn;
    }
    float ss = 0.f;
    for (int d = lane; d < hd; d += 32) {
        const float v = bf16_bits_to_f32(p[d]);
        t[d] = v;
        ss += v * v;
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)hd + a.eps);
    for (int d = lane; d < hd; d += 32) t[d] = t[d] * inv * g[d];  // each lane its own elements
    __syncwarp();
    const float* cs = a.rope_cos + (size_t)pos * hd;
    const float* sn = a.rope_sin + (size_t)pos * hd;
    for (int d = lane; d < hd; d += 32) {
        const float rot = d < half ? -t[d + half] : t[d - half];
        p[d] = f32_to_bf16_bits(t[d] * cs[d] + rot * sn[d]);
    }
}

cudaError_t launch_qk_norm(const QkNormArgs& a, bool pdl, cudaStream_t st) {
    if (a.hd > kAttnMaxHd || a.hd % 2 || a.M < 1) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(a.nq + a.n_kv, a.M);
    cfg.blockDim = dim3(32);
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_qk_norm, a);
}

// ----------------------------------------------------------------- embed --
__global__ void __launch_bounds__(256) k_embed(EmbedArgs a) {
    const int m = blockIdx.x;
    pdl_wait();
    pdl_launch();
    int slot, pos;
    uint32_t id;
    if (a.mode == 0) {
        slot = m;
        pos = a.pos[m];
        id = a.ids_ring[(size_t)(*a.step) * a.batch + m];
    } else {
        slot = a.slot;
        pos = a.pos[a.slot] + m;
        id = a.prefill_ids[m];
    }
    if (id >= (uint32_t)a.vocab) {
        // host ids are checked before the launch; a device id (the caller's
        // seeds of decode_device) is reported through the error word, and
        // the gather never reads out of range
        if (threadIdx.x == 0) atomicCAS(a.err, 0, RENG_E_INVAL);
        id = 0;
    }
    if (threadIdx.x == 0) {
        a.row_slot[m] = slot;
        a.row_pos[m] = pos;
    }
    const uint4* src = reinterpret_cast<const uint4*>(a.table + (size_t)id * a.hidden);
    uint4* dst = reinterpret_cast<uint4*>(a.x_res + (size_t)m * a.hidden);
    const int nv = a.hidden / 8;  // hidden % 16 == 0: pairs of chunks are whole tiles
    for (int base = 0; base < nv; base += blockDim.x) {
        const int i = base + threadIdx.x;
        float ss = 0.f;
        if (i < nv) {
            uint4 v = ldg_nc(src + i);
            dst[i] = v;
            float t[8] = {bf16lo(v.x), bf16hi(v.x), bf16lo(v.y), bf16hi(v.y),
                          bf16lo(v.z), bf16hi(v.z), bf16lo(v.w), bf16hi(v.w)};
#pragma unroll
            for (int e = 0; e < 8; e++) ss += t[e] * t[e];
        }
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        if (i < nv && (i & 1) == 0) a.ss_out[(size_t)m * kSsStride + (i >> 1)] = ss;
    }
}

cudaError_t launch_embed(const EmbedArgs& a, bool pdl, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(a.M);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_embed, a);
}

// ------------------------------------------------------------------ pack --
// bf16 packing: one thread per 16-byte piece of a block: atom a, row r,
// stored chunk position p holding logical chunk j = p ^ r (k = 64c + 8j).
__global__ void k_pack(PackArgs a) {
    const int64_t total = (int64_t)a.tiles * a.kc * 128;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int p = (int)(i & 7), r = (int)((i >> 3) & 7), at = (int)((i >> 6) & 1);
        const int64_t blk = i >> 7;
        const int c = (int)(blk % a.kc);
        const int tile = (int)(blk / a.kc);
        const int srow = a.rowmap[tile * kTileRows + at * 8 + r];
        const int k0 = c * kChunkK + ((p ^ r) & 7) * 8;
        uint16_t v[8];
#pragma unroll
        for (int e = 0; e < 8; e++) {
            uint16_t b = 0;
            if (srow >= 0 && k0 + e < a.K) {
                b = a.src[(int64_t)srow * a.ld + k0 + e];
                if (a.scale != 0.0f && srow < a.scale_rows)
                    b = f32_to_bf16_bits(bf16_bits_to_f32(b) * a.scale);
            }
            v[e] = b;
        }
        uint4 o;
        o.x = v[0] | ((uint32_t)v[1] << 16);
        o.y = v[2] | ((uint32_t)v[3] << 16);
        o.z = v[4] | ((uint32_t)v[5] << 16);
        o.w = v[6] | ((uint32_t)v[7] << 16);
        *reinterpret_cast<uint4*>(a.dst + blk * kBlockBytesBf16 + at * 1024 + r * 128 + p * 16) = o;
    }
}

cudaError_t launch_pack(const PackArgs& a, cudaStream_t st) {
    const int64_t total = (int64_t)a.tiles * a.kc * 128;
    int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 32);
    k_pack<<<grid, 256, 0, st>>>(a);
    return cudaGetLastError();
}

// FP8 packing: one thread per (block, half, lane) 16-byte piece: row 8h + l/4
// of the tile, k = 64c + 16(l%4) .. +16.
__global__ void k_pack8(Pack8Args a) {
    const int64_t total = (int64_t)a.tiles * a.kc * 64;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int lane = (int)(i & 31), h = (int)((i >> 5) & 1);
        const int64_t blk = i >> 6;
        const int c = (int)(blk % a.kc);
        const int tile = (int)(blk / a.kc);
        const int srow = a.rowmap[tile * kTileRows + h * 8 + (lane >> 2)];
        const int k0 = c * 64 + (lane & 3) * 16;
        uint8_t v[16];
#pragma unroll
        for (int e = 0; e < 16; e++) v[e] = (srow >= 0 && k0 + e < a.K) ? a.src[(int64_t)srow * a.K + k0 + e] : 0;
        uint4 o;
        o.x = v[0] | (v[1] << 8) | (v[2] << 16) | ((uint32_t)v[3] << 24);
        o.y = v[4] | (v[5] << 8) | (v[6] << 16) | ((uint32_t)v[7] << 24);
        o.z = v[8] | (v[9] << 8) | (v[10] << 16) | ((uint32_t)v[11] << 24);
        o.w = v[12] | (v[13] << 8) | (v[14] << 16) | ((uint32_t)v[15] << 24);
        *reinterpret_cast<uint4*>(a.dst + blk * kBlockBytesFp8 + h * 512 + lane * 16) = o;
    }
}

cudaError_t launch_pack8(const Pack8Args& a, cudaStream_t st) {
    const int64_t total = (int64_t)a.tiles * a.kc * 64;
    int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 32);
    k_pack8<<<grid, 256, 0, st>>>(a);
    return cudaGetLastError();
}

// Row scales in packed row order: dst[p] = src[rowmap[p]] (x mul for the
// rows below mul_rows: the attention scale on the q rows); 0 for padding.
__global__ void k_gather_scales(const float* src, const int* rowmap, int n, float mul, int mul_rows, float* dst) {
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < n; p += gridDim.x * blockDim.x) {
        const int r = rowmap[p];
        dst[p] = r < 0 ? 0.f : (r < mul_rows ? src[r] * mul : src[r]);
    }
}

cudaError_t launch_gather_scales(const float* src, const int* rowmap, int n, float mul, int mul_rows, float* dst,
                                 cudaStream_t st) {
    k_gather_scales<<<(n + 255) / 256, 256, 0, st>>>(src, rowmap, n, mul, mul_rows, dst);
    return cudaGetLastError();
}

__global__ void k_bf16_to_f32(const uint16_t* s, float* d, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        d[i] = bf16_bits_to_f32(s[i]);
}

cudaError_t launch_bf16_to_f32(const uint16_t* src, float* dst, int64_t n, cudaStream_t st) {
    int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
    if (grid < 1) grid = 1;
    k_bf16_to_f32<<<grid, 256, 0, st>>>(src, dst, n);
    return cudaGetLastError();
}

}  // namespace reng
