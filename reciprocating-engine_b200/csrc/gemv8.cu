// Packed-weight GEMV for 2..8 activation rows with the x fragments held in
// registers (decode at batch 2..8).
//
// The shared-memory GEMV (decode.cu) stages the x rows in each CTA: at 8
// rows of 4096 that is 66 KB, which leaves one 8-warp CTA per SM with a
// 128 KB weight ring.  Here each warp owns a fixed k-range of BPW packed
// blocks (kc = 8 * BPW), so a lane needs only the x values its MMAs read
// for that range: 8 u32 per block (64 registers at BPW = 8).  They are
// loaded once, RMS-normalised in registers, and the weight ring takes all
// of shared memory: 8 warps x 6 stages x 4 KB = 192 KB in flight per SM,
// as at batch 1 (three 4-warp CTAs of 4 stages).
//
// Staging: before the wait on the previous kernel each warp issues 3 of its
// 6 ring stages and one bulk copy brings the RMSNorm gains (constants) into
// shared memory.  After the wait, x row m is bulk-copied into stages 3..5
// of warp m's ring (its weight copies are not issued yet) and the rows'
// norm partials into the reduction buffer; the lanes build their fragments,
// and the three stages then join the weight stream.  The chunk loop over a
// tile's blocks is unrolled so the fragments stay in registers.
#include <algorithm>

#include "gemv_core.cuh"

namespace reng {

namespace {

constexpr int kW8Warps = 8;                   // warps per CTA (one CTA per SM)
constexpr int kW8Stages = 6;                  // ring stages per warp
constexpr int kW8XStage = 3;                  // first stage of the x-row staging
constexpr int kW8MaxK = (kW8Stages - kW8XStage) * kChunkBytes / 2;  // x row in 3 stages: 6144 bf16
constexpr int kW8Ring = kW8Stages * kChunkBytes;                    // bytes per warp

// One block's MMAs from register fragments.  bf16: xr[0] = row g, k = 32h +
// 8q .. +8 for h = 0, xr[1] for h = 1 (the shared-memory path's
// x_fragment).  FP8: xr[0], xr[1] = row g, k = 16q .. +16 as f16 (its
// x_fragment16).
template <int W8>
__device__ __forceinline__ void block_mma_reg(float (&acc)[4], const uint4 (&v)[4], const uint4& x0, const uint4& x1) {
    if (!W8) {
        mma_bf16_16816(acc, v[0].x, v[2].x, v[0].y, v[2].y, x0.x, x0.y);
        mma_bf16_16816(acc, v[0].z, v[2].z, v[0].w, v[2].w, x0.z, x0.w);
        mma_bf16_16816(acc, v[1].x, v[3].x, v[1].y, v[3].y, x1.x, x1.y);
        mma_bf16_16816(acc, v[1].z, v[3].z, v[1].w, v[3].w, x1.z, x1.w);
    } else {
        const uint32_t ra[4] = {v[0].x, v[0].y, v[0].z, v[0].w}, rb[4] = {v[1].x, v[1].y, v[1].z, v[1].w};
        const uint32_t xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int i = 0; i < 4; i++)
            mma_f16_16816(acc, e4m3x2_to_f16x2(ra[i] & 0xffffu), e4m3x2_to_f16x2(rb[i] & 0xffffu),
                          e4m3x2_to_f16x2(ra[i] >> 16), e4m3x2_to_f16x2(rb[i] >> 16), xv[2 * i], xv[2 * i + 1]);
    }
}

// 8 staged bf16 values (row g, k .. k + 8) -> the lane's fragment word set:
// normalised with inv * gain[k + i] when gains are given, as bf16 (bf16
// weights) or f16 (FP8 weights).
template <int W8>
__device__ __forceinline__ uint4 make_frag(uint4 v, float inv, const float* gain) {
    float t[8] = {bf16lo(v.x), bf16hi(v.x), bf16lo(v.y), bf16hi(v.y), bf16lo(v.z), bf16hi(v.z), bf16lo(v.w), bf16hi(v.w)};
    if (gain != nullptr) {
#pragma unroll
        for (int i = 0; i < 8; i++) t[i] = t[i] * inv * gain[i];
    }
    if (W8)
        return make_uint4(pack_f16x2(t[0], t[1]), pack_f16x2(t[2], t[3]), pack_f16x2(t[4], t[5]), pack_f16x2(t[6], t[7]));
    if (gain == nullptr) return v;
    return make_uint4(pack_bf16x2(t[0], t[1]), pack_bf16x2(t[2], t[3]), pack_bf16x2(t[4], t[5]), pack_bf16x2(t[6], t[7]));
}

}  // namespace

template <int EPI, int W8, int BPW>
__global__ void __launch_bounds__(kW8Warps * 32, 1) k_gemv8(GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem_dyn[];
    constexpr int BB = W8 ? kBlockBytesFp8 : kBlockBytesBf16;  // bytes per block
    constexpr int CB = kChunkBytes / BB;                        // blocks per chunk
    constexpr int NCT = (BPW + CB - 1) / CB;                    // chunks per tile per warp
    constexpr int NP = W8 ? 2 : 4;                              // 16-byte pieces per lane per block
    __shared__ __align__(16) float4 red_buf[kMaxRows * 256 / 4];  // tile reduction / RMS partials
    __shared__ __align__(16) float gains[kW8MaxK];
    __shared__ float inv_s[kMaxRows];
    __shared__ int s_ids[kMaxRows];
    __shared__ int s_last;
    __shared__ __align__(8) unsigned long long bars[kW8Warps * kW8Stages];
    __shared__ __align__(8) unsigned long long xbar, gbar;
    float4(*red)[32] = reinterpret_cast<float4(*)[32]>(red_buf);
    const int K = a.K;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const int c0 = warp * BPW;  // this warp's blocks [c0, c0 + BPW) of every tile
    int poff[4];
    lane_pieces<W8>(g, q, lane, poff);
    const int ntile = blockIdx.x < a.tiles ? (a.tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int nchunks = ntile * NCT;
    const bool norm = a.ss_in != nullptr;

    const uint32_t ring = (uint32_t)__cvta_generic_to_shared(smem_dyn) + warp * kW8Ring;
    const uint32_t bar0 = (uint32_t)__cvta_generic_to_shared(&bars[0]) + warp * kW8Stages * 8;
    const uint32_t xbar_a = (uint32_t)__cvta_generic_to_shared(&xbar);
    const uint32_t gbar_a = (uint32_t)__cvta_generic_to_shared(&gbar);
    bool failed = false;
    int issued = 0, waited = 0;
    auto tma_issue = [&](int j) {  // lane 0 only: chunk j of this warp's sequence
        if (j >= nchunks || failed) return;
        const int tile = blockIdx.x + (j / NCT) * gridDim.x;
        const int b0 = (j % NCT) * CB;
        const int nb = min(CB, BPW - b0);
        const uint32_t bar = bar0 + (j % kW8Stages) * 8;
        mbar_expect_tx(bar, (uint32_t)(nb * BB));
        tma_load_1d(ring + (j % kW8Stages) * kChunkBytes, a.w + ((size_t)tile * a.kc + c0 + b0) * BB,
                    (uint32_t)(nb * BB), bar);
        issued = j + 1;
    };
    if (threadIdx.x == 0) {
        mbar_init(xbar_a, 1);
        mbar_init(gbar_a, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        if (norm) {  // the gains are constants: before the wait
            mbar_expect_tx(gbar_a, (uint32_t)(K * 4));
            tma_load_1d((uint32_t)__cvta_generic_to_shared(gains), a.gain, (uint32_t)(K * 4), gbar_a);
        }
    }
    if (lane == 0) {
        for (int s2 = 0; s2 < kW8Stages; s2++) mbar_init(bar0 + s2 * 8, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int j = 0; j < kW8XStage; j++) tma_issue(j);
    }
    __syncwarp();

    pdl_wait();
    pdl_launch();

    // x row m into stages 3..5 of warp m's ring, the RMS partials into the
    // reduction buffer (one bulk copy each)
    __syncthreads();  // barrier inits visible to every thread before any wait
    const bool ss_tma = norm && (a.ss_tiles & 3) == 0 && a.M * a.ss_tiles * 4 <= (int)sizeof(red_buf);
    if (threadIdx.x == 0) {
        const uint32_t ssb = (uint32_t)(a.ss_tiles * 4);
        mbar_expect_tx(xbar_a, (uint32_t)(a.M * K * 2) + (ss_tma ? a.M * ssb : 0u));
        for (int m = 0; m < a.M; m++)
            tma_load_1d((uint32_t)__cvta_generic_to_shared(smem_dyn) + m * kW8Ring + kW8XStage * kChunkBytes,
                        a.x + (size_t)m * a.ldx, (uint32_t)(K * 2), xbar_a);
        if (ss_tma)
            for (int m = 0; m < a.M; m++)
                tma_load_1d((uint32_t)__cvta_generic_to_shared(red_buf) + m * ssb, a.ss_in + (size_t)m * kSsStride,
                            ssb, xbar_a);
    }
    if (norm && !ss_tma && warp < a.M) {  // partials too many for the buffer: plain loads
        float s = 0.0f;
        for (int t = lane; t < a.ss_tiles; t += 32) s += a.ss_in[(size_t)warp * kSsStride + t];
        s = warp_sum(s);
        if (lane == 0) inv_s[warp] = 1.0f / sqrtf(s / (float)a.norm_k + a.eps);
    }
    if (!mbar_wait_bounded(xbar_a, 0) || (norm && !mbar_wait_bounded(gbar_a, 0))) {
        failed = true;
        if (lane == 0) atomicExch(a.err, RENG_E_TIMEOUT);
    }
    if (ss_tma && warp < a.M) {
        const float4* sp = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(red_buf) + warp * a.ss_tiles);
        float s = 0.0f;
        for (int t = lane; t < a.ss_tiles / 4; t += 32) {
            const float4 v = sp[t];
            s += (v.x + v.y) + (v.z + v.w);
        }
        s = warp_sum(s);
        if (lane == 0) inv_s[warp] = 1.0f / sqrtf(s / (float)a.norm_k + a.eps);
    }
    __syncthreads();
    // this lane's fragments: row g of its warp's k-range
    uint4 xr[BPW][2];
    {
        const uint16_t* xrow =
            reinterpret_cast<const uint16_t*>(smem_dyn + g * kW8Ring + kW8XStage * kChunkBytes);
        const float inv = g < a.M && norm ? inv_s[g] : 1.0f;
#pragma unroll
        for (int b = 0; b < BPW; b++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                // bf16: k = 64c + 32h + 8q; FP8: k = 64c + 16q + 8h
                const int k = (c0 + b) * kChunkK + (W8 ? q * 16 + h * 8 : h * 32 + q * 8);
                if (g < a.M && k < K)
                    xr[b][h] = make_frag<W8>(*reinterpret_cast<const uint4*>(xrow + k), inv, norm ? gains + k : nullptr);
                else
                    xr[b][h] = make_uint4(0u, 0u, 0u, 0u);
            }
    }
    __syncthreads();  // every lane has read the staged rows
    __syncwarp();
    if (lane == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int j = kW8XStage; j < kW8Stages; j++) tma_issue(j);
    }
    __syncwarp();

    float best_v[2] = {-INFINITY, -INFINITY};
    int best_i[2] = {0, 0};
    int j = 0;
    for (int it = 0; it < ntile; it++) {
        const int tile = blockIdx.x + it * gridDim.x;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int cc = 0; cc < NCT; cc++, j++) {
            const uint32_t bar = bar0 + (j % kW8Stages) * 8;
            if (!failed) {
                if (mbar_wait_bounded(bar, (uint32_t)((j / kW8Stages) & 1))) {
                    waited = j + 1;
                } else {
                    failed = true;
                    if (lane == 0) atomicExch(a.err, RENG_E_TIMEOUT);
                }
            }
            const uint32_t st = ring + (j % kW8Stages) * kChunkBytes;
#pragma unroll
            for (int i = 0; i < CB; i++) {
                const int b = cc * CB + i;
                if (b < BPW) {
                    uint4 v[4];
#pragma unroll
                    for (int p = 0; p < NP; p++) v[p] = lds128(st + i * BB + poff[p]);
                    block_mma_reg<W8>(acc, v, xr[b][0], xr[b][1]);
                }
            }
            // the stage is read: let the async proxy refill it
            __syncwarp();
            if (lane == 0) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                tma_issue(j + kW8Stages);
            }
            __syncwarp();
        }
        // ---- the tile is complete: reduce the warps' k-slices on warp 0 ----
        __syncthreads();
        red[warp][lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        __syncthreads();
        if (warp == 0) {
#pragma unroll
            for (int w = 1; w < kW8Warps; w++) {
                const float4 r = red[w][lane];
                acc[0] += r.x;
                acc[1] += r.y;
                acc[2] += r.z;
                acc[3] += r.w;
            }
            if (W8) {  // per-row scale of the FP8 codes
                const float s0 = a.wscale[tile * kTileRows + g], s1 = a.wscale[tile * kTileRows + g + 8];
                acc[0] *= s0;
                acc[1] *= s0;
                acc[2] *= s1;
                acc[3] *= s1;
            }
            gemv_epilogue<EPI>(a, tile, acc, g, q, best_v, best_i);
        }
    }
    if (failed && lane == 0) {
        // drain this warp's own copies still in flight before exiting (bounded)
        for (int jj = waited; jj < issued; jj++)
            if (!mbar_wait_bounded(bar0 + (jj % kW8Stages) * 8, (uint32_t)((jj / kW8Stages) & 1))) break;
    }

    if (EPI == EPI_LOGITS) {
        // this CTA's best per row into the rows' running maxima; the last
        // CTA reads them out (as the shared-memory GEMV's LM head)
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

namespace {
template <int EPI, int W8, int BPW>
cudaError_t launch8(const GemvArgs& a, bool pdl, cudaStream_t st) {
    static_assert(kW8Warps * kW8Ring <= 200 * 1024, "ring");
    int dev = 0;
    cudaGetDevice(&dev);
    const int grid = std::min(a.tiles, num_sms(dev));
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kW8Warps * 32);
    cfg.dynamicSmemBytes = kW8Warps * kW8Ring;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_gemv8<EPI, W8, BPW>, a);
}

template <int EPI, int BPW>
cudaError_t launch8_w(const GemvArgs& a, bool pdl, cudaStream_t st) {
    return a.w8 ? launch8<EPI, 1, BPW>(a, pdl, st) : launch8<EPI, 0, BPW>(a, pdl, st);
}

template <int EPI>
cudaError_t launch8_b(const GemvArgs& a, bool pdl, cudaStream_t st) {
    return a.kc == 8 * kW8Warps ? launch8_w<EPI, 8>(a, pdl, st) : launch8_w<EPI, 10>(a, pdl, st);
}

template <int EPI, int W8, int BPW>
cudaError_t prepare8() {
    return cudaFuncSetAttribute(k_gemv8<EPI, W8, BPW>, cudaFuncAttributeMaxDynamicSharedMemorySize, kW8Warps * kW8Ring);
}

template <int EPI>
cudaError_t prepare8_e() {
    cudaError_t e = prepare8<EPI, 0, 8>();
    if (e == cudaSuccess) e = prepare8<EPI, 1, 8>();
    if (e == cudaSuccess) e = prepare8<EPI, 0, 10>();
    if (e == cudaSuccess) e = prepare8<EPI, 1, 10>();
    return e;
}
}  // namespace

// Whether the register-fragment GEMV runs this projection: 2..8 rows, every
// warp the same k-range of 8 or 10 packed blocks (K of 4096 or 5120), an x
// row within three ring stages.
bool gemv8_fits(const GemvArgs& a) {
    // from 2 rows: measured on B200 (Llama-8B), b2 4.47 -> 4.07 ms per step;
    // at 1 row the 444-CTA shared-memory GEMV stays ahead (3.20 against 3.36)
    static const int min_rows = [] {  // RENG_GEMV8_MIN_ROWS: a tuning knob (1..8)
        const char* v = getenv("RENG_GEMV8_MIN_ROWS");
        const int x = v ? atoi(v) : 0;
        return x >= 1 && x <= kMaxRows ? x : 2;
    }();
    return a.M >= min_rows && a.M <= kMaxRows && (a.kc == 8 * kW8Warps || a.kc == 10 * kW8Warps) &&
           a.K <= kW8MaxK && a.K % 8 == 0 && a.kc * kChunkK >= a.K;
}

cudaError_t gemv8_prepare() {
    cudaError_t e = prepare8_e<EPI_QKV>();
    if (e == cudaSuccess) e = prepare8_e<EPI_RESID>();
    if (e == cudaSuccess) e = prepare8_e<EPI_SWIGLU>();
    if (e == cudaSuccess) e = prepare8_e<EPI_LOGITS>();
    if (e == cudaSuccess) e = prepare8_e<EPI_F32>();
    return e;
}

cudaError_t launch_gemv8(const GemvArgs& a, int epi, bool pdl, cudaStream_t st) {
    if (!gemv8_fits(a)) return cudaErrorInvalidValue;
    switch (epi) {
        case EPI_QKV: return launch8_b<EPI_QKV>(a, pdl, st);
        case EPI_RESID: return launch8_b<EPI_RESID>(a, pdl, st);
        case EPI_SWIGLU: return launch8_b<EPI_SWIGLU>(a, pdl, st);
        case EPI_LOGITS: return launch8_b<EPI_LOGITS>(a, pdl, st);
        case EPI_F32: return launch8_b<EPI_F32>(a, pdl, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace reng
