// Device pieces of the packed-weight GEMV (decode.cu, and gemv8.cu / gemm.cu
// for the primitives): the x fragments of the m16n8k16 MMAs, one packed
// block into the accumulators, the tile epilogues, and the mbarrier /
// bulk-copy primitives of the per-warp TMA weight rings.
#pragma once
#include "decode.cuh"

namespace reng {

// The x fragment of lane (g, q) for k-chunk c: row g, k = 32c + 8q .. +8,
// as 4 u32 of packed bf16.  From the CTA's shared copy when it was staged,
// else straight from global memory (rows too long for shared memory; only
// un-normalised inputs take that path).
__device__ __forceinline__ uint4 x_fragment(const GemvArgs& a, const uint16_t* xs, int xstride,
                                            int K, int c, int h, int g, int q) {
    const int k = c * kChunkK + h * 32 + q * 8;
    if (g >= a.M || k >= K) return make_uint4(0u, 0u, 0u, 0u);
    if (xs != nullptr) return *reinterpret_cast<const uint4*>(xs + g * xstride + k);
    return ldg_nc(a.x + (size_t)g * a.ldx + k);
}

// RMS-normalise the staged x rows in place: x' = bf16(x * inv[m] * gain[k])
// (f16 for the FP8-weight kernels, whose mma runs in f16).
template <int W8>
__device__ __forceinline__ void normalise_x(const GemvArgs& a, uint16_t* xs, int xstride, int K,
                                            const float* inv_s) {
    const int nv = K / 8;
    for (int i = threadIdx.x; i < a.M * nv; i += blockDim.x) {
        const int m = i / nv, k = (i % nv) * 8;
        uint4* p = reinterpret_cast<uint4*>(xs + m * xstride + k);
        uint4 v = *p;
        const float inv = inv_s[m];
        const float4 g0 = __ldg(reinterpret_cast<const float4*>(a.gain + k));
        const float4 g1 = __ldg(reinterpret_cast<const float4*>(a.gain + k + 4));
        if (W8) {
            v.x = pack_f16x2(bf16lo(v.x) * inv * g0.x, bf16hi(v.x) * inv * g0.y);
            v.y = pack_f16x2(bf16lo(v.y) * inv * g0.z, bf16hi(v.y) * inv * g0.w);
            v.z = pack_f16x2(bf16lo(v.z) * inv * g1.x, bf16hi(v.z) * inv * g1.y);
            v.w = pack_f16x2(bf16lo(v.w) * inv * g1.z, bf16hi(v.w) * inv * g1.w);
        } else {
            v.x = pack_bf16x2(bf16lo(v.x) * inv * g0.x, bf16hi(v.x) * inv * g0.y);
            v.y = pack_bf16x2(bf16lo(v.y) * inv * g0.z, bf16hi(v.y) * inv * g0.w);
            v.z = pack_bf16x2(bf16lo(v.z) * inv * g1.x, bf16hi(v.z) * inv * g1.y);
            v.w = pack_bf16x2(bf16lo(v.w) * inv * g1.z, bf16hi(v.w) * inv * g1.w);
        }
        *p = v;
    }
}

// The same with the gains already in registers: thread t owns the 8-wide
// k-groups t + j * blockDim.x (j < GV), loaded before the kernel waited on
// its predecessor (the gains are constants), so the normalisation after
// the wait costs no global round trip.
template <int GV>
__device__ __forceinline__ void gain_preload(const GemvArgs& a, int K, float4 (&gp)[GV][2]) {
    const int nv = K / 8;
#pragma unroll
    for (int j = 0; j < GV; j++) {
        const int kv = threadIdx.x + j * blockDim.x;
        if (kv < nv) {
            gp[j][0] = __ldg(reinterpret_cast<const float4*>(a.gain) + 2 * kv);
            gp[j][1] = __ldg(reinterpret_cast<const float4*>(a.gain) + 2 * kv + 1);
        }
    }
}

template <int W8, int GV>
__device__ __forceinline__ void normalise_x_pre(const GemvArgs& a, uint16_t* xs, int xstride, int K,
                                                const float* inv_s, const float4 (&gp)[GV][2]) {
    const int nv = K / 8;
#pragma unroll
    for (int j = 0; j < GV; j++) {
        const int kv = threadIdx.x + j * blockDim.x;
        if (kv >= nv) continue;
        const float4 g0 = gp[j][0], g1 = gp[j][1];
        for (int m = 0; m < a.M; m++) {
            uint4* p = reinterpret_cast<uint4*>(xs + m * xstride + kv * 8);
            uint4 v = *p;
            const float inv = inv_s[m];
            if (W8) {
                v.x = pack_f16x2(bf16lo(v.x) * inv * g0.x, bf16hi(v.x) * inv * g0.y);
                v.y = pack_f16x2(bf16lo(v.y) * inv * g0.z, bf16hi(v.y) * inv * g0.w);
                v.z = pack_f16x2(bf16lo(v.z) * inv * g1.x, bf16hi(v.z) * inv * g1.y);
                v.w = pack_f16x2(bf16lo(v.w) * inv * g1.z, bf16hi(v.w) * inv * g1.w);
            } else {
                v.x = pack_bf16x2(bf16lo(v.x) * inv * g0.x, bf16hi(v.x) * inv * g0.y);
                v.y = pack_bf16x2(bf16lo(v.y) * inv * g0.z, bf16hi(v.y) * inv * g0.w);
                v.z = pack_bf16x2(bf16lo(v.z) * inv * g1.x, bf16hi(v.z) * inv * g1.y);
                v.w = pack_bf16x2(bf16lo(v.w) * inv * g1.z, bf16hi(v.w) * inv * g1.w);
            }
            *p = v;
        }
    }
}

// Staged bf16 x rows -> f16 in place (FP8-weight kernels without a norm).
__device__ __forceinline__ void x_to_f16(const GemvArgs& a, uint16_t* xs, int xstride, int K) {
    const int nv = K / 8;
    for (int i = threadIdx.x; i < a.M * nv; i += blockDim.x) {
        const int m = i / nv, k = (i % nv) * 8;
        uint4* p = reinterpret_cast<uint4*>(xs + m * xstride + k);
        uint4 v = *p;
        v.x = bf16x2_to_f16x2(v.x);
        v.y = bf16x2_to_f16x2(v.y);
        v.z = bf16x2_to_f16x2(v.z);
        v.w = bf16x2_to_f16x2(v.w);
        *p = v;
    }
}

// FP8 blocks: lane (g, q) multiplies k = 64c + 16q .. +16; its x fragment is
// those 16 values of row g as f16 (two uint4).
__device__ __forceinline__ void x_fragment16(const GemvArgs& a, const uint16_t* xs, int xstride, int K, int c,
                                             int g, int q, uint4& lo, uint4& hi) {
    const int k = c * 64 + q * 16;
    if (g >= a.M || k >= K) {
        lo = hi = make_uint4(0u, 0u, 0u, 0u);
        return;
    }
    if (xs != nullptr) {
        lo = *reinterpret_cast<const uint4*>(xs + g * xstride + k);
        hi = *reinterpret_cast<const uint4*>(xs + g * xstride + k + 8);
        return;
    }
    const uint4 b0 = ldg_nc(a.x + (size_t)g * a.ldx + k), b1 = ldg_nc(a.x + (size_t)g * a.ldx + k + 8);
    lo = make_uint4(bf16x2_to_f16x2(b0.x), bf16x2_to_f16x2(b0.y), bf16x2_to_f16x2(b0.z), bf16x2_to_f16x2(b0.w));
    hi = make_uint4(bf16x2_to_f16x2(b1.x), bf16x2_to_f16x2(b1.y), bf16x2_to_f16x2(b1.z), bf16x2_to_f16x2(b1.w));
}

// One packed block into the accumulators.  bf16: two m16n8k16 steps over
// 32 k.  FP8: the lane's 16 codes of rows g and g+8 become f16 pairs and run
// four f16 steps over 64 k; step i takes codes 4i..4i+3 (k pairs (2q, 2q+1)
// and (2q+8, 2q+9) of the step in the mma's numbering), matched by the same
// x values.
template <int W8>
__device__ __forceinline__ void block_mma(float (&acc)[4], const uint4 (&v)[4], const GemvArgs& a,
                                          const uint16_t* xs, int xstride, int K, int c, int g, int q) {
    if (!W8) {
        // v: row g (k-half 0, 1), row g+8 (k-half 0, 1)
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint4 xf = x_fragment(a, xs, xstride, K, c, h, g, q);
            mma_bf16_16816(acc, v[h].x, v[2 + h].x, v[h].y, v[2 + h].y, xf.x, xf.y);
            mma_bf16_16816(acc, v[h].z, v[2 + h].z, v[h].w, v[2 + h].w, xf.z, xf.w);
        }
    } else {
        // v[0]: 16 codes of row g, v[1]: of row g+8
        uint4 xl, xh;
        x_fragment16(a, xs, xstride, K, c, g, q, xl, xh);
        const uint32_t ra[4] = {v[0].x, v[0].y, v[0].z, v[0].w}, rb[4] = {v[1].x, v[1].y, v[1].z, v[1].w};
        const uint32_t xv[8] = {xl.x, xl.y, xl.z, xl.w, xh.x, xh.y, xh.z, xh.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            mma_f16_16816(acc, e4m3x2_to_f16x2(ra[i] & 0xffffu), e4m3x2_to_f16x2(rb[i] & 0xffffu),
                          e4m3x2_to_f16x2(ra[i] >> 16), e4m3x2_to_f16x2(rb[i] >> 16), xv[2 * i], xv[2 * i + 1]);
        }
    }
}

// Byte offsets, inside a block, of lane (g, q)'s 16-byte pieces in the order
// block_mma takes them.
template <int W8>
__device__ __forceinline__ void lane_pieces(int g, int q, int lane, int (&off)[4]) {
    if (!W8) {
        off[0] = g * 128 + ((q ^ g) & 7) * 16;                 // row g, k 8q (chunk q)
        off[1] = g * 128 + (((4 + q) ^ g) & 7) * 16;           // row g, k 32 + 8q (chunk 4 + q)
        off[2] = 1024 + off[0];                               // row g + 8: same swizzle phase
        off[3] = 1024 + off[1];
    } else {
        off[0] = lane * 16;
        off[1] = 512 + lane * 16;
        off[2] = off[3] = 0;
    }
}

// Lexicographic argmax step: larger value, then lower index.
// The reference's fold (strict '>' from -inf, index 0 when nothing beats
// -inf): NaN and -inf are never taken, equal values keep the first index.
__device__ __forceinline__ void am_take(float& bv, int& bi, float v, int i) {
    if (v > bv || (v == bv && i < bi && v > -INFINITY)) {
        bv = v;
        bi = i;
    }
}

__device__ __forceinline__ void am_reduce_g(float& bv, int& bi) {
    // across the 8 lanes that share q (xor over the g bits 2,3,4 of the lane id)
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        am_take(bv, bi, ov, oi);
    }
}


// The epilogue of one 16-row tile on one warp: acc holds rows {g, g+8} x
// activation rows {2q, 2q+1}.  x_res and the row bookkeeping are read
// through L2 (ld.global.cg), not the SM's incoherent L1.
template <int EPI>
__device__ __forceinline__ void gemv_epilogue(const GemvArgs& a, int tile, const float (&acc)[4], int g,
                                              int q, float (&best_v)[2], int (&best_i)[2]) {
    // ---- epilogue (warp 0): acc = rows {g, g+8} x cols {2q, 2q+1} ----
    const int m0 = 2 * q, m1 = 2 * q + 1;
    if (EPI == EPI_RESID) {
        const int r0 = tile * kTileRows + g, r1 = r0 + 8;
        float s0 = 0.f, s1 = 0.f;
        if (m0 < a.M) {
            uint16_t* o = a.out + (size_t)m0 * a.ldo;
            float x0 = round_bf16(bf16_bits_to_f32(__ldcg(o + r0)) + round_bf16(acc[0]));
            float x1 = round_bf16(bf16_bits_to_f32(__ldcg(o + r1)) + round_bf16(acc[2]));
            o[r0] = f32_to_bf16_bits(x0);
            o[r1] = f32_to_bf16_bits(x1);
            s0 = x0 * x0 + x1 * x1;
        }
        if (m1 < a.M) {
            uint16_t* o = a.out + (size_t)m1 * a.ldo;
            float x0 = round_bf16(bf16_bits_to_f32(__ldcg(o + r0)) + round_bf16(acc[1]));
            float x1 = round_bf16(bf16_bits_to_f32(__ldcg(o + r1)) + round_bf16(acc[3]));
            o[r0] = f32_to_bf16_bits(x0);
            o[r1] = f32_to_bf16_bits(x1);
            s1 = x0 * x0 + x1 * x1;
        }
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            s0 += __shfl_xor_sync(0xffffffffu, s0, o);
            s1 += __shfl_xor_sync(0xffffffffu, s1, o);
        }
        if (g == 0) {
            if (m0 < a.M) a.ss_out[(size_t)m0 * kSsStride + tile] = s0;
            if (m1 < a.M) a.ss_out[(size_t)m1 * kSsStride + tile] = s1;
        }
    } else if (EPI == EPI_F32) {
        const int r0 = tile * kTileRows + g, r1 = r0 + 8;
        if (m0 < a.M) {
            a.out_f32[(size_t)m0 * a.ldo + r0] = acc[0];
            a.out_f32[(size_t)m0 * a.ldo + r1] = acc[2];
        }
        if (m1 < a.M) {
            a.out_f32[(size_t)m1 * a.ldo + r0] = acc[1];
            a.out_f32[(size_t)m1 * a.ldo + r1] = acc[3];
        }
    } else if (EPI == EPI_SWIGLU) {
        const int j = tile * 8 + g;
        if (m0 < a.M) {
            float gt = acc[0], up = acc[2];
            a.out[(size_t)m0 * a.ldo + j] = f32_to_bf16_bits(gt / (1.0f + expf(-gt)) * up);
        }
        if (m1 < a.M) {
            float gt = acc[1], up = acc[3];
            a.out[(size_t)m1 * a.ldo + j] = f32_to_bf16_bits(gt / (1.0f + expf(-gt)) * up);
        }
    } else if (EPI == EPI_QKV) {
        const int hd = a.head_dim, half = hd >> 1, ppt = hd >> 4;  // pair tiles per head
        const int q_dim = (a.q_tiles / ppt) * hd, kv_dim = a.n_kv * hd;
        if (tile < a.q_tiles + a.k_tiles) {
            const bool is_q = tile < a.q_tiles;
            const int t = is_q ? tile : tile - a.q_tiles;
            const int h = t / ppt, d = (t % ppt) * 8 + g, d2 = d + half;
            const int brow = is_q ? h * hd : q_dim + h * hd;
            float b1 = a.bias ? a.bias[brow + d] : 0.f, b2 = a.bias ? a.bias[brow + d2] : 0.f;
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int m = e ? m1 : m0;
                if (m >= a.M) continue;
                const int pos = __ldcg(a.row_pos + m);
                if (pos >= a.cap) continue;
                float x1 = (e ? acc[1] : acc[0]) + b1;
                float x2 = (e ? acc[3] : acc[2]) + b2;
                const float* cs = a.rope_cos + (size_t)pos * hd;
                const float* sn = a.rope_sin + (size_t)pos * hd;
                float y1 = x1 * cs[d] - x2 * sn[d];
                float y2 = x2 * cs[d2] + x1 * sn[d2];
                if (is_q) {
                    uint16_t* o = a.out + (size_t)m * a.ldo + h * hd;
                    o[d] = f32_to_bf16_bits(y1);
                    o[d2] = f32_to_bf16_bits(y2);
                } else {
                    const int slot = __ldcg(a.row_slot + m);
                    uint16_t* kc = a.kcache + (((size_t)slot * a.n_kv + h) * a.cap + pos) * hd;
                    kc[d] = f32_to_bf16_bits(y1);
                    kc[d2] = f32_to_bf16_bits(y2);
                }
            }
        } else {
            const int vt = tile - a.q_tiles - a.k_tiles;
#pragma unroll
            for (int rr = 0; rr < 2; rr++) {
                const int r = vt * kTileRows + g + rr * 8;
                const int h = r / hd, d = r % hd;
                const float b = a.bias ? a.bias[q_dim + kv_dim + r] : 0.f;
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const int m = e ? m1 : m0;
                    if (m >= a.M) continue;
                    const int pos = __ldcg(a.row_pos + m);
                    if (pos >= a.cap) continue;
                    const int slot = __ldcg(a.row_slot + m);
                    float val = acc[rr * 2 + e] + b;
                    a.vcache[(((size_t)slot * a.n_kv + h) * a.cap + pos) * hd + d] =
                        f32_to_bf16_bits(val);
                }
            }
        }
    } else if (EPI == EPI_LOGITS) {
        const int r0 = a.row0 + tile * kTileRows + g, r1 = r0 + 8;  // global vocabulary rows
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const int m = e ? m1 : m0;
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            if (m < a.M) {
                if (r0 < a.vocab) {
                    uint16_t b = f32_to_bf16_bits(acc[e]);
                    a.out[(size_t)m * a.ldo + r0] = b;
                    am_take(bv, bi, bf16_bits_to_f32(b), r0);
                }
                if (r1 < a.vocab) {
                    uint16_t b = f32_to_bf16_bits(acc[2 + e]);
                    a.out[(size_t)m * a.ldo + r1] = b;
                    am_take(bv, bi, bf16_bits_to_f32(b), r1);
                }
            }
            am_reduce_g(bv, bi);
            am_take(best_v[e], best_i[e], bv, bi);
        }
    }
}

// ---- weight pipelines ----------------------------------------------------
// Each warp walks a flat sequence of chunks (its k-range of a tile, tile
// after tile of the CTA) so the stream never restarts at a tile boundary.
//
// Each warp owns a ring of stages of kChunkBytes of contiguous packed
// blocks in shared memory (kTmaStages of them), filled by
// one cp.async.bulk (TMA) copy per stage and an mbarrier with the
// transaction byte count; lane 0 refills a stage as soon as the warp has
// read it.  Every mbarrier wait is bounded by a %globaltimer deadline: on
// expiry the kernel records RENG_E_TIMEOUT in *a.err, stops issuing
// copies, drains its own copies (again bounded) and finishes without
// waiting.
constexpr int kChunkBytes = 4096;                             // weight bytes per pipeline chunk
constexpr int kTmaStages = 4;
constexpr unsigned long long kWaitNs = 2000000000ull;           // 2 s per wait

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: false if the deadline passed first.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(bar, parity))
        if (globaltimer() - t0 > kWaitNs) return false;
    return true;
}
__device__ __forceinline__ void tma_load_1d(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// 16-byte store / load of two 64-bit words, each single-copy atomic, that
// bypass the non-coherent caches (peer memory written over NVLink).
__device__ __forceinline__ void st_words(unsigned long long* p, unsigned long long a, unsigned long long b) {
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_words(const unsigned long long* p, unsigned long long& a, unsigned long long& b) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Sharded LM head: this rank's argmax key of row m pushed to every peer,
// the peers' keys of row m collected (bounded wait on their epoch words),
// the maximum returned.  The maximum of am_pack keys is the largest value
// with the smallest global index, so every rank gets the replicated head's
// id.  Every calling thread reads the same epoch; the caller advances it
// once all have finished.
__device__ __forceinline__ unsigned long long head_exchange(const HeadXchg* hx, int m, unsigned long long key,
                                                            int* err) {
    const unsigned e = *reinterpret_cast<const volatile unsigned*>(hx->epoch) + 1;
    const size_t par = (size_t)(e & 1) * kTpMaxWorld * kMaxRows * 2;
    const unsigned long long w0 = ((unsigned long long)e << 32) | (key >> 32);
    const unsigned long long w1 = ((unsigned long long)e << 32) | (key & 0xffffffffull);
    for (int r = 0; r < hx->world; r++)
        if (r != hx->rank) st_words(hx->recv[r] + par + ((size_t)hx->rank * kMaxRows + m) * 2, w0, w1);
    unsigned long long best = key;
    for (int r = 0; r < hx->world; r++) {
        if (r == hx->rank) continue;
        const unsigned long long* src = hx->recv[hx->rank] + par + ((size_t)r * kMaxRows + m) * 2;
        unsigned long long a, b;
        ld_words(src, a, b);
        if ((a >> 32) != e || (b >> 32) != e) {
            const unsigned long long t0 = globaltimer();
            do {
                ld_words(src, a, b);
                if (globaltimer() - t0 > kWaitNs) {
                    atomicExch(err, RENG_E_TIMEOUT);
                    return best;
                }
            } while ((a >> 32) != e || (b >> 32) != e);
        }
        const unsigned long long k = ((a & 0xffffffffull) << 32) | (b & 0xffffffffull);
        if (k > best) best = k;
    }
    return best;
}

__device__ __forceinline__ uint4 lds128(uint32_t saddr) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(saddr));
    return r;
}


}  // namespace reng
