// tcgen05 / TMEM GEMM for steps with many activation rows (batch > 8 decode
// and prefill blocks): Y[m, row] = sum_k X[m, k] * W[row, k] with the
// weights as the MMA's A operand (M = 128 weight rows per tile) and the
// activation rows as its N (16..256), so a wide batch is one N dimension and
// the weights stream from HBM once per step.
//
// Operands in shared memory use the K-major 128-byte-swizzle atom of the
// UMMA descriptors (8 rows x 128 B, 16-byte chunk j of row r at j ^ r):
//  * A (weights): the packed blocks are already that atom, so a stage is
//    eight 2 KB bulk copies (one per 16-row tile of the 128-row super-tile);
//  * B (activations, row-major [rows][K] bf16): a 2-D tensor-map copy with
//    128-byte swizzle of a {64 k, N rows} box.
// Both give SBO = 1024 B (one 8-row atom), and the K=16 steps inside a
// 64-k stage advance the descriptor start address by 32 B.
//
// Scheduling (k_gemm_sk): persistent stream-K.  One CTA per SM takes an
// equal share of the (super-tile, 64-k chunk) work in super-tile-major
// order, so every SM streams weights from its first chunk to its last
// whatever the matrix shape (a 4096-row projection has 32 super-tiles, a
// Llama LM head 1002).  Roles (192 threads): warp 0 lane 0 issues the
// copies into an up-to-8-stage ring, warp 1 owns the TMEM accumulators (two
// buffers of N f32 columns) and lane 0 issues tcgen05.mma.kind::f16 and
// commits each stage back to the producer and each finished segment to the
// epilogue, warps 2-5 read TMEM with tcgen05.ld (warp w: lanes 32*(w%4) ..
// +32) and apply the same epilogues as the GEMV kernels while the next
// segment accumulates in the other buffer.  Super-tiles split between two
// or more shares are finished by the last of their CTAs to arrive, which
// adds the f32 partials in K order.  Every mbarrier wait is bounded.
#include <mutex>
#include <string>
#include <vector>

#include "gemm.cuh"
#include "gemv_core.cuh"

namespace reng {

namespace {

constexpr int kGemmThreads = 192;
constexpr int kGemmMaxStages = 8;  // pipeline stages (runtime: GemmArgs::stages)
constexpr int kGemmStageBudget = 200 * 1024;                  // stage bytes of a one-per-SM launch
constexpr int kGemmMaxDynSmem = kGemmStageBudget + 2048;      // + the 1024-byte alignment slack
constexpr int kStageA = 8 * kBlockBytesBf16;  // 128 rows x 64 k
constexpr unsigned long long kGemmWaitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void bar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool bar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity) {
    if (bar_try(bar, parity)) return true;
    const unsigned long long t0 = gtimer();
    while (!bar_try(bar, parity))
        if (gtimer() - t0 > kGemmWaitNs) return false;
    return true;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tensor_g2s(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tensor_g2s_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z,
                                              uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tensor_g2s_4d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, int w,
                                              uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar)
        : "memory");
}
// UMMA shared-memory descriptor: K-major, 128-byte swizzle, SBO 1024 B.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset: next 8-row atom
    d |= (uint64_t)1 << 46;             // descriptor version (sm100)
    d |= (uint64_t)2 << 61;             // SWIZZLE_128B
    return d;
}
// Instruction descriptor: f32 accumulate, bf16 A and B, both K-major, M=128.
__device__ __forceinline__ uint32_t umma_idesc(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
__device__ __forceinline__ void umma(uint32_t tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void named_sync_epilogue() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ void am_take2(float& bv, int& bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

}  // namespace

// Epilogue of 16 activation columns (m = cb*16 .. +16) of one weight row
// (packed row p of the matrix, TMEM lane `lr` of the super-tile).
template <int EPI>
__device__ __forceinline__ void tc_epilogue16(const GemmArgs& g, int p, int lr, int cb, const float (&v)[16],
                                              float* am_v, int* am_i, int warp_e) {
    const GemvArgs& a = g.e;
    const int lane = lr & 31;
    const int tile = p >> 4, i16 = p & 15;
    // rows past the matrix (the last 16-row tile, the last 128-row CTA
    // tile) are computed but never stored
    const bool valid = tile < g.tiles16 && (EPI == EPI_SWIGLU || EPI == EPI_QKV || EPI == EPI_LOGITS || p < a.ldo);
    // every global load of the 16 columns is issued before the arithmetic
    // that needs it (one round trip per group, not one per column)
    if (EPI == EPI_RESID) {
        uint16_t xo[16];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const int m = cb * 16 + j;
            xo[j] = (valid && m < a.M) ? __ldcg(a.out + (size_t)m * a.ldo + p) : (uint16_t)0;
        }
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const int m = cb * 16 + j;
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
            const int m = cb * 16 + j;
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
            const int m = cb * 16 + j;
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
        const int m = cb * 16 + j;
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
            if (lane == 0) {
                am_v[warp_e * kRowsCap + m] = bv;
                am_i[warp_e * kRowsCap + m] = bi;
            }
        }
    }
}

// The CTA's share of the launch's work: chunks [start, end) of the
// super-tile-major chunk order (super-tile S owns chunks S*kc .. S*kc+kc-1),
// start = floor(c * T / G) for CTA c of G and T chunks in all.
__device__ __forceinline__ long long sk_start(long long c, long long T, long long G) { return c * T / G; }
// The CTA whose share holds chunk x: the largest c with sk_start(c) <= x.
__device__ __forceinline__ int sk_owner(long long x, long long T, long long G) {
    return (int)(((x + 1) * G - 1) / T);
}
// Partial-tile slot of CTA c's segment of super-tile S: a share holds at
// most two split super-tiles, the one it starts in (slot 2c) and the one it
// ends in (slot 2c + 1).
__device__ __forceinline__ int sk_slot(int c, int S, int kc, long long T, long long G) {
    return (int)(sk_start(c, T, G) / kc) == S ? 2 * c : 2 * c + 1;
}

// The copy units of a CTA's share: runs of up to C consecutive chunks of
// one segment (one super-tile), each fetched by one weight copy and one
// activation copy into one pipeline stage.
struct SkUnits {
    long long x, x0, x1;
    int kc, C;
    __device__ bool next(int& S, int& c0, int& cnt, bool& first, bool& last) {
        if (x >= x1) return false;
        S = (int)(x / kc);
        c0 = (int)(x % kc);
        const long long seg0 = max(x0, (long long)S * kc), seg1 = min(x1, (long long)(S + 1) * kc);
        cnt = (int)min((long long)C, seg1 - x);
        first = x == seg0;
        last = x + cnt == seg1;
        x += cnt;
        return true;
    }
};

// LM-head argmax of one finished super-tile: the 4 epilogue warps' best per
// row into the rows' running maxima; the CTA that finishes the launch's last
// super-tile reads the keys, swaps them with the other ranks (vocabulary
// shards) and writes the ids.
__device__ __forceinline__ void sk_logits_tile_done(const GemmArgs& g, float* am_v, int* am_i, int* s_done) {
    const GemvArgs& a = g.e;
    named_sync_epilogue();
    for (int m = threadIdx.x - 64; m < a.M; m += 128) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int w = 0; w < 4; w++) am_take2(bv, bi, am_v[w * kRowsCap + m], am_i[w * kRowsCap + m]);
        atomicMax(a.am_key + m, am_pack(bv, bi));
    }
    __threadfence();
    named_sync_epilogue();
    if (threadIdx.x == 64) *s_done = (atomicAdd(a.am_count, 1u) == (unsigned)g.super_tiles - 1);
    named_sync_epilogue();
    if (*s_done) {
        __threadfence();
        for (int m = threadIdx.x - 64; m < a.M; m += 128) {
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
    named_sync_epilogue();  // am_v / am_i are free for the next super-tile
}

// Persistent stream-K GEMM: one CTA per SM, each streaming an equal share
// of the launch's (super-tile, 64-k chunk) work in super-tile-major order,
// so every SM keeps weights in flight from its first chunk to its last,
// whatever the matrix's shape.  A share is a run of segments (one
// super-tile's chunks each); a segment accumulates in one of two TMEM
// buffers, so the epilogue warps finish segment j while the MMA warp fills
// the other buffer with segment j + 1 and the producer streams on.  A
// segment that covers its super-tile's whole K runs the epilogue from TMEM;
// a split super-tile's segments store f32 partials, and the last of its
// CTAs to arrive adds them in K order (deterministic: the same sum whoever
// arrives last) and runs the epilogue.  Every mbarrier wait is bounded.
template <int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1) k_gemm_sk(const __grid_constant__ CUtensorMap tmap_x,
                                                             const __grid_constant__ CUtensorMap tmap_w, GemmArgs g) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ __align__(8) unsigned long long full[kGemmMaxStages], empty[kGemmMaxStages], acc_full[2],
        acc_empty[2], drain;
    __shared__ uint32_t tmem_base_s;
    __shared__ int s_flag, s_done;
    __shared__ float am_v[EPI == EPI_LOGITS ? 4 * kRowsCap : 1];
    __shared__ int am_i[EPI == EPI_LOGITS ? 4 * kRowsCap : 1];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x;
    const long long G = gridDim.x, T = (long long)g.super_tiles * g.kc;
    const long long x0 = sk_start(c, T, G), x1 = sk_start(c + 1, T, G);
    const int kc = g.kc, N = g.N, SG = g.stages, C = g.C;
    const uint32_t stage_bytes = (uint32_t)C * (kStageA + (uint32_t)N * 128u);
    const uint32_t b_off = (uint32_t)C * kStageA;  // the stage's activation tiles follow its C weight tiles
    const uint32_t smem0 = ((uint32_t)__cvta_generic_to_shared(smem_raw) + 1023u) & ~1023u;
    const uint32_t bar_full = (uint32_t)__cvta_generic_to_shared(&full[0]);
    const uint32_t bar_empty = (uint32_t)__cvta_generic_to_shared(&empty[0]);
    const uint32_t bar_accf = (uint32_t)__cvta_generic_to_shared(&acc_full[0]);
    const uint32_t bar_acce = (uint32_t)__cvta_generic_to_shared(&acc_empty[0]);
    const uint32_t bar_drain = (uint32_t)__cvta_generic_to_shared(&drain);
    // two accumulators of N columns, each at a power-of-two column offset
    uint32_t half = 16;
    while ((int)half < N) half <<= 1;
    const uint32_t ncols = half < 16 ? 32 : 2 * half;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SG; s++) {
            bar_init(bar_full + 8 * s, 1);
            bar_init(bar_empty + 8 * s, 1);
        }
        for (int b = 0; b < 2; b++) {
            bar_init(bar_accf + 8 * b, 1);
            bar_init(bar_acce + 8 * b, 4);  // lane 0 of each epilogue warp
        }
        bar_init(bar_drain, 1);
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

    if (warp == 0) {
        if (lane == 0) {
            // one weight copy (C chunks x 8 tiles x 2 KB, rows past the
            // matrix and chunks past K read as zeros) and one activation copy
            // (or one per chunk when K is ragged) per unit
            const uint32_t tx_b = (uint32_t)N * 128u;
            auto issue_a = [&](int i, int S, int c0) {
                tensor_g2s_4d(smem0 + (uint32_t)(i % SG) * stage_bytes, &tmap_w, 0, 0, 8 * S, c0,
                              bar_full + 8 * (i % SG));
            };
            auto issue_b = [&](int i, int c0, int cnt) {
                const uint32_t dst = smem0 + (uint32_t)(i % SG) * stage_bytes + b_off;
                if (g.b3d) {
                    tensor_g2s_3d(dst, &tmap_x, 0, 0, c0, bar_full + 8 * (i % SG));
                } else {
                    for (int q = 0; q < cnt; q++)
                        tensor_g2s(dst + (uint32_t)q * tx_b, &tmap_x, (c0 + q) * kChunkK, 0, bar_full + 8 * (i % SG));
                }
            };
            auto tx_of = [&](int cnt) { return (uint32_t)C * kStageA + (uint32_t)(g.b3d ? C : cnt) * tx_b; };
            SkUnits ua{x0, x0, x1, kc, C}, ub{x0, x0, x1, kc, C};
            int S, c0, cnt, i = 0;
            bool first, last;
            // the weights do not depend on the previous kernel
            while (i < SG && ua.next(S, c0, cnt, first, last)) {
                bar_expect_tx(bar_full + 8 * i, tx_of(cnt));
                issue_a(i, S, c0);
                i++;
            }
            const int pre = i;
            pdl_wait();
            for (int k = 0; k < pre && ub.next(S, c0, cnt, first, last); k++) issue_b(k, c0, cnt);
            int issued = pre;
            while (ua.next(S, c0, cnt, first, last)) {
                const int s = i % SG;
                if (!bar_wait(bar_empty + 8 * s, (uint32_t)(((i / SG) - 1) & 1))) {
                    atomicExch(g.e.err, RENG_E_TIMEOUT);
                    break;
                }
                bar_expect_tx(bar_full + 8 * s, tx_of(cnt));
                issue_a(i, S, c0);
                issue_b(i, c0, cnt);
                issued = ++i;
            }
            // the last copy into each stage has landed before the CTA may
            // exit (already true unless a wait gave up; bounded)
            for (int k = max(0, issued - SG); k < issued; k++)
                if (!bar_wait(bar_full + 8 * (k % SG), (uint32_t)((k / SG) & 1))) atomicExch(g.e.err, RENG_E_TIMEOUT);
        } else {
            pdl_wait();
        }
        pdl_launch();
    } else if (warp == 1) {
        pdl_wait();
        pdl_launch();
        if (lane == 0) {
            const uint32_t idesc = umma_idesc(N);
            SkUnits u{x0, x0, x1, kc, C};
            int S, c0, cnt, i = 0, j = -1, b = 0;
            bool first, last;
            uint32_t acc = tmem;
            while (u.next(S, c0, cnt, first, last)) {
                if (first) {
                    b = ++j & 1;
                    if (j >= 2 && !bar_wait(bar_acce + 8 * b, (uint32_t)(((j / 2) - 1) & 1))) {
                        atomicExch(g.e.err, RENG_E_TIMEOUT);
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    acc = tmem + (uint32_t)b * half;
                }
                const int s = i % SG;
                if (!bar_wait(bar_full + 8 * s, (uint32_t)((i / SG) & 1))) {
                    atomicExch(g.e.err, RENG_E_TIMEOUT);
                    umma_commit(bar_accf + 8 * b);  // the epilogue then sees the error word
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t st0 = smem0 + (uint32_t)s * stage_bytes;
                for (int q = 0; q < cnt; q++) {
                    const uint32_t a0 = st0 + (uint32_t)q * kStageA, b0 = st0 + b_off + (uint32_t)q * (uint32_t)N * 128u;
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        umma(acc, umma_desc(a0 + kk * 32), umma_desc(b0 + kk * 32), idesc,
                             (first && q == 0 && kk == 0) ? 0u : 1u);
                }
                umma_commit(bar_empty + 8 * s);
                i++;
                if (last) umma_commit(bar_accf + 8 * b);  // fires when this segment's MMAs have finished
            }
            // every MMA this thread issued has completed before TMEM is freed
            umma_commit(bar_drain);
            if (!bar_wait(bar_drain, 0)) atomicExch(g.e.err, RENG_E_TIMEOUT);
        }
    } else {
        // ---- epilogue warps 2..5: TMEM lanes 32 * (warp % 4) .. +32 ----
        pdl_wait();
        pdl_launch();
        const int q4 = warp & 3, warp_e = warp - 2;
        const int lr = 32 * q4 + lane;
        const int ncb = N / 16;
        int j = 0;
        for (long long x = x0; x < x1; j++) {
            const int S = (int)(x / kc), kb = (int)(x % kc), ke = (int)min((long long)kc, kb + (x1 - x));
            x += ke - kb;
            const int b = j & 1;
            const int p = 128 * S + lr;  // packed row of the matrix
            if (!bar_wait(bar_accf + 8 * b, (uint32_t)((j / 2) & 1))) {
                if (lane == 0) atomicExch(g.e.err, RENG_E_TIMEOUT);
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t trow = tmem + ((uint32_t)(32 * q4) << 16) + (uint32_t)b * half;
            if (kb == 0 && ke == kc) {
                // the whole K of this super-tile: epilogue straight from TMEM
                for (int cb = 0; cb < ncb; cb++) {
                    float v[16];
                    tmem_ld16(trow + cb * 16, v);
                    tc_epilogue16<EPI>(g, p, lr, cb, v, am_v, am_i, warp_e);
                }
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) bar_arrive(bar_acce + 8 * b);
                if (EPI == EPI_LOGITS) sk_logits_tile_done(g, am_v, am_i, &s_done);
                continue;
            }
            // a split super-tile: this share's partial to its slot,
            // [slot][cb][128 rows][16] f32 (a warp stores 2 KB contiguous)
            const int slot = sk_slot(c, S, kc, T, G);
            float* mine = g.gpart + (size_t)slot * ncb * 128 * 16;
            for (int cb = 0; cb < ncb; cb++) {
                float v[16];
                tmem_ld16(trow + cb * 16, v);
                float4* dst = reinterpret_cast<float4*>(mine + ((size_t)cb * 128 + lr) * 16);
#pragma unroll
                for (int q = 0; q < 4; q++) __stcg(dst + q, make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) bar_arrive(bar_acce + 8 * b);
            const int cf = sk_owner((long long)S * kc, T, G), cl = sk_owner((long long)S * kc + kc - 1, T, G);
            __threadfence();
            named_sync_epilogue();
            if (threadIdx.x == 64) s_flag = atomicAdd(g.gcnt + S, 1) == cl - cf;
            named_sync_epilogue();
            if (!s_flag) continue;
            // the last CTA of this super-tile: every share's partial, in K
            // order; the loads of up to 4 shares go out together (one L2
            // round trip per 4 shares and column group, not one per share)
            __threadfence();
            for (int cb = 0; cb < ncb; cb++) {
                float v[16];
#pragma unroll
                for (int q = 0; q < 16; q++) v[q] = 0.f;
                for (int c4 = cf; c4 <= cl; c4 += 4) {
                    float4 t4[4][4];
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const int cc = min(c4 + u, cl);
                        const float4* src = reinterpret_cast<const float4*>(
                            g.gpart + ((size_t)sk_slot(cc, S, kc, T, G) * ncb * 128 + (size_t)cb * 128 + lr) * 16);
#pragma unroll
                        for (int q = 0; q < 4; q++) t4[u][q] = __ldcg(src + q);
                    }
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        if (c4 + u > cl) break;
#pragma unroll
                        for (int q = 0; q < 4; q++) {
                            v[4 * q] += t4[u][q].x;
                            v[4 * q + 1] += t4[u][q].y;
                            v[4 * q + 2] += t4[u][q].z;
                            v[4 * q + 3] += t4[u][q].w;
                        }
                    }
                }
                tc_epilogue16<EPI>(g, p, lr, cb, v, am_v, am_i, warp_e);
            }
            if (threadIdx.x == 64) g.gcnt[S] = 0;
            if (EPI == EPI_LOGITS) sk_logits_tile_done(g, am_v, am_i, &s_done);
        }
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

size_t gemm_smem_bytes(int n, int stages, int c) { return (size_t)stages * c * (kStageA + (size_t)n * 128) + 1024; }

int gemm_chunks_per_stage(int n) { return n <= 128 ? 2 : 1; }

int gemm_pick_stages(int n, int c) {
    // One CTA per SM: as many stages as fit the ~200 KB budget (8 at N <= 64:
    // 128 KB of weights in flight per SM; 4 at N = 256).  RENG_GEMM_STAGES
    // caps it (a tuning knob).
    static const int cap = [] {
        const char* v = getenv("RENG_GEMM_STAGES");
        const int x = v ? atoi(v) : 0;
        return x >= 2 && x <= kGemmMaxStages ? x : kGemmMaxStages;
    }();
    int s = (int)((unsigned)kGemmStageBudget / ((unsigned)c * (kStageA + (unsigned)n * 128u)));
    if (s > cap) s = cap;
    return s < 2 ? 2 : s;
}

void gemm_plan(int super_tiles, int kc, int n, int sms, int* grid, int* stages, int* c) {
    // Fewer super-tiles than SMs (the 4096-row projections: 32): ks CTAs
    // per super-tile, so each is split in ks shares (about kc / ks chunks)
    // that finish together and whose partials the last CTA reads in one go;
    // at N >= 128 at most 2 (a 128 x N partial is 64-128 KB, as large as 4-8
    // chunks of weights).  Otherwise one CTA per SM, each super-tile split
    // in at most 2-3 shares.
    long long G;
    if (super_tiles >= sms) {
        G = sms;
    } else {
        int ks = sms / super_tiles;
        static const int cap_env = [] {  // RENG_GEMM_KS: a tuning knob for the shares cap
            const char* v = getenv("RENG_GEMM_KS");
            const int x = v ? atoi(v) : 0;
            return x >= 1 && x <= 8 ? x : 0;
        }();
        const int cap = cap_env ? cap_env : (n >= 128 ? 2 : 4);
        if (ks > cap) ks = cap;
        if (ks > kc) ks = kc;
        if (ks < 1) ks = 1;
        G = (long long)super_tiles * ks;
    }
    const long long T = (long long)super_tiles * kc;
    *grid = (int)(T < G ? T : G);
    *c = gemm_chunks_per_stage(n);
    *stages = gemm_pick_stages(n, *c);
}

size_t gemm_scratch_floats(int grid, int n) { return (size_t)2 * grid * n * 128; }

template <int EPI>
static cudaError_t launch_tc_t(const CUtensorMap& map, const CUtensorMap& wmap, const GemmArgs& g, bool pdl,
                               cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(g.grid);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = gemm_smem_bytes(g.N, g.stages, g.C);
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_gemm_sk<EPI>, map, wmap, g);
}

template <int EPI>
static cudaError_t prepare_t() {
    return cudaFuncSetAttribute(k_gemm_sk<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmMaxDynSmem);
}

cudaError_t gemm_prepare() {
    cudaError_t e = prepare_t<EPI_QKV>();
    if (e == cudaSuccess) e = prepare_t<EPI_RESID>();
    if (e == cudaSuccess) e = prepare_t<EPI_SWIGLU>();
    if (e == cudaSuccess) e = prepare_t<EPI_LOGITS>();
    if (e == cudaSuccess) e = prepare_t<EPI_F32>();
    return e;
}

cudaError_t launch_gemm_tc(const CUtensorMap& map, const CUtensorMap& wmap, const GemmArgs& g, int epi, bool pdl,
                           cudaStream_t st) {
    const long long T = (long long)g.super_tiles * g.kc;
    if (g.N % 16 || g.N < 16 || g.N > kRowsCap || g.e.M > g.N || g.e.M < 1 || g.grid < 1 || g.grid > T ||
        g.C < 1 || g.C > 4 || g.stages < 2 || g.stages > kGemmMaxStages ||
        gemm_smem_bytes(g.N, g.stages, g.C) > (size_t)kGemmMaxDynSmem || g.gpart == nullptr || g.gcnt == nullptr ||
        g.super_tiles > kGemmCntMax || (g.b3d && g.kc * kChunkK != g.e.K))
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
    RENG_CHECK_ARG(M >= 1 && M <= kRowsCap, "reng_gemm_bf16: M must be in [1, 256]");
    RENG_CHECK_ARG(splits >= -8 && splits <= 8 && iters >= 0 && (iters == 0 || ms_out),
                   "reng_gemm_bf16: bad splits / iters");
    RENG_CHECK_ARG(mem == RENG_MEM_HOST || mem == RENG_MEM_DEVICE, "reng_gemm_bf16: bad mem");
    const cudaMemcpyKind h2d = mem == RENG_MEM_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
    const cudaMemcpyKind d2h = mem == RENG_MEM_HOST ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
    int dev = 0;
    GEMM_CU(cudaGetDevice(&dev));
    GEMM_CU(gemm_prepare());
    const int tiles = (rows + kTileRows - 1) / kTileRows, kc = (K + kChunkK - 1) / kChunkK;
    const int N = (M + 15) / 16 * 16;
    DevFree f;
    uint16_t *wd = nullptr, *xd = nullptr;
    uint8_t* packed = nullptr;
    int* rowmap = nullptr;
    float* yd = nullptr;
    int* err = nullptr;
    GEMM_CU(f.alloc(&wd, (size_t)rows * K * 2));
    GEMM_CU(f.alloc(&xd, (size_t)kRowsCap * K * 2));
    GEMM_CU(f.alloc(&packed, (size_t)tiles * kc * kBlockBytesBf16));
    GEMM_CU(f.alloc(&rowmap, (size_t)tiles * kTileRows * 4));
    GEMM_CU(f.alloc(&yd, (size_t)M * rows * 4));
    GEMM_CU(f.alloc(&err, 4));
    GEMM_CU(cudaMemcpy(wd, w, (size_t)rows * K * 2, h2d));
    GEMM_CU(cudaMemset(xd, 0, (size_t)kRowsCap * K * 2));
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
    gemm_plan(g.super_tiles, kc, N, num_sms(dev), &g.grid, &g.stages, &g.C);
    if (splits != 0) {
        // that many CTAs per super-tile (capped by the chunks and the SMs):
        // shares that split super-tiles in several ways, for checks
        const long long T = (long long)g.super_tiles * kc;
        long long want = (long long)g.super_tiles * (splits > 0 ? splits : -splits);
        if (want > T) want = T;
        if (want > num_sms(dev)) want = num_sms(dev);
        g.grid = (int)want;
    }
    GEMM_CU(f.alloc(&g.gpart, gemm_scratch_floats(g.grid, N) * 4));
    GEMM_CU(f.alloc(&g.gcnt, (size_t)g.super_tiles * 4));
    GEMM_CU(cudaMemset(g.gcnt, 0, (size_t)g.super_tiles * 4));
    CUtensorMap tmap, wmap;
    g.b3d = K % kChunkK == 0;
    int rc = g.b3d ? gemm_tensor_map3(xd, kRowsCap, K, N, g.C, &tmap) : gemm_tensor_map(xd, kRowsCap, K, N, &tmap);
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
