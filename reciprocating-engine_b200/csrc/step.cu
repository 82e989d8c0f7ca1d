// The persistent decode step: the embedding gather, every layer's five
// phases (q/k/v + RoPE + KV write, attention, o_proj + residual, gate/up +
// SwiGLU, down_proj + residual) and the LM head with its argmax, as phases
// of ONE cooperative launch (one CTA per SM, 12 warps).  The reference runs
// the same op sequence as one SynapseAI recipe per step
// (crates/reng-synapse/src/cached.rs:752-835, model.rs:1172-1944).
//
// Why one launch: with a kernel per projection every launch pays a ramp
// (CTAs scheduled, barriers set up, the first weight bytes in flight) and a
// drain (the slowest CTA), several microseconds each, against 5-40 us of
// useful weight streaming.  Here each warp owns a TMA ring (4 KB slots) fed
// from ONE sequence of weight chunks that runs through all the projections
// of the step in order: weights never depend on activations, so while a
// warp waits at a phase boundary (a grid barrier) or works on attention,
// its ring already holds the next projection's first chunks.
//
// Work split (stream-K): a projection is T = tiles x kc packed blocks; warp
// w of the G' = min(G, T) warps takes blocks [w*T/G', (w+1)*T/G') of the
// tile-major order, so every warp streams the same number of bytes.  A
// warp's partial sums of a tile it shares with others go to a global slot;
// the warp that arrives last at the tile (counter) adds the slots in warp
// order (deterministic) and runs the tile epilogue (the same epilogues as
// the per-projection kernels).  Attention: a CTA per (row, KV group, key
// range) with the keys staged in shared memory, the last CTA of a (row,
// group) combining the ranges in order.
//
// The phase table lives in global memory; each phase's arguments are copied
// to shared memory when the phase starts (the inner loops read them there),
// and the chunk cursors keep their phase's constants in registers.
//
// Waits: the grid barrier, the ring and the x staging waits are bounded by
// %globaltimer; on expiry the CTA records RENG_E_TIMEOUT and sets *abort, and
// every later barrier falls through, so the launch always ends.
#include "gemv_core.cuh"
#include "step.cuh"

namespace reng {

namespace {

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ int ld_volatile_i32(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// Grid-wide barrier closing phase p: one atomic per CTA on a 64-bit arrival
// count that only grows (every launch adds the same multiple of the grid),
// so the count returned by the arrival names the barrier's target.
__device__ void grid_sync(const StepCtl& c, int p) {
    __syncthreads();
    if (threadIdx.x == 0) {
        if (c.trace != nullptr) {
            const unsigned long long t = globaltimer();
            atomicMin(c.trace + kTraceStride * p + 1, t);
            atomicMax(c.trace + kTraceStride * p + 2, t);
        }
        if (ld_volatile_i32(c.abort) == 0) {
            __threadfence();
            const unsigned long long nb = gridDim.x;
            const unsigned long long old = atomicAdd(c.bar, 1ull);
            const unsigned long long target = (old / nb + 1) * nb;
            if (old + 1 != target) {
                const unsigned long long t0 = globaltimer();
                while (ld_acquire_u64(c.bar) < target) {
                    if (ld_volatile_i32(c.abort)) break;
                    if (globaltimer() - t0 > kWaitNs) {
                        atomicExch(c.abort, 1);
                        atomicExch(c.err, RENG_E_TIMEOUT);
                        break;
                    }
                }
            }
            __threadfence();
        }
        if (blockIdx.x == 0 && c.trace != nullptr) c.trace[kTraceStride * (p + 1)] = globaltimer();
    }
    __syncthreads();
}

// The CTAs taking part in a phase of T blocks: all C, or T when there are
// fewer blocks than CTAs (one block each), so every range is non-empty.
__device__ __forceinline__ int phase_ctas(long long T, int C) { return T < C ? (int)T : C; }

// The CTA that owns block b when T blocks are split over C (<= T) CTAs.
__device__ __forceinline__ int block_owner(long long b, long long T, int C) { return (int)(((b + 1) * C - 1) / T); }

// A CTA's contiguous block range [lo, hi) of a phase (T blocks over the
// phase's CTAs); empty (lo == hi) for CTAs past them.
__device__ __forceinline__ void cta_range(long long T, int C, int b, int& lo, int& hi) {
    const int Cp = phase_ctas(T, C);
    if (b >= Cp) {
        lo = hi = 0;
        return;
    }
    lo = (int)((long long)b * T / Cp);
    hi = (int)((long long)(b + 1) * T / Cp);
}

// Warp w's share [s0, s1) of tile t's blocks in the CTA range [lo, hi):
// the range's part of the tile split evenly over the warps.
__device__ __forceinline__ void warp_share(int lo, int hi, int kc, int t, int w, int& s0, int& s1) {
    const int a0 = max(lo, t * kc), a1 = min(hi, (t + 1) * kc), len = a1 - a0;
    s0 = a0 + w * len / kStepWarps;
    s1 = a0 + (w + 1) * len / kStepWarps;
}

// A warp's position in the step's weight-chunk sequence (its shares of
// every tile of its CTA's range, phase after phase), with the phase's
// constants in registers.
struct Cursor {
    int p;               // phase (nph: past the end)
    int kc, bb;          // blocks per tile, bytes per block
    int lo, hi;          // the CTA's range
    int tile;            // current tile
    int pos, end;        // current block, end of the warp's share of the tile
    const uint8_t* w;    // the phase's packed weights
};

__device__ void cursor_fix(const StepSeq* seq, int nph, Cursor& k, int cta, int C, int warp);

// The first GEMV phase >= p in which this warp has blocks.
__device__ void cursor_seek(const StepSeq* seq, int nph, Cursor& k, int p, int cta, int C, int warp) {
    for (; p < nph; p++) {
        const StepSeq q = seq[p];
        if (q.blocks == 0) continue;
        int lo, hi;
        cta_range(q.blocks, C, cta, lo, hi);
        if (lo == hi) continue;
        k.p = p;
        k.kc = q.kc;
        k.bb = q.bb;
        k.w = q.w;
        k.lo = lo;
        k.hi = hi;
        k.tile = lo / k.kc;
        warp_share(lo, hi, k.kc, k.tile, warp, k.pos, k.end);
        cursor_fix(seq, nph, k, cta, C, warp);
        return;
    }
    k.p = nph;
}

// Past an empty share: the next tile of the range, or the next phase.
__device__ void cursor_fix(const StepSeq* seq, int nph, Cursor& k, int cta, int C, int warp) {
    while (k.pos == k.end) {
        if (k.tile >= (k.hi - 1) / k.kc) {
            cursor_seek(seq, nph, k, k.p + 1, cta, C, warp);
            return;
        }
        k.tile++;
        warp_share(k.lo, k.hi, k.kc, k.tile, warp, k.pos, k.end);
    }
}

// Blocks in the chunk at the cursor: at most one ring slot, within one share.
__device__ __forceinline__ int cursor_chunk(const Cursor& k) { return min(kStepChunk / k.bb, k.end - k.pos); }

__device__ __forceinline__ const uint8_t* cursor_src(const Cursor& k) { return k.w + (size_t)k.pos * k.bb; }

__device__ __forceinline__ void cursor_advance(const StepSeq* seq, int nph, Cursor& k, int n, int cta, int C,
                                               int warp) {
    k.pos += n;
    cursor_fix(seq, nph, k, cta, C, warp);
}

__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// The blocks of one ring slot into four accumulators (two per block parity,
// split by k half or by MMA parity) so that consecutive MMAs do not wait on
// each other.  xl: the lane's x row offset by its k within a block, cst the
// row's bytes per block (0 for the lanes past the rows, which read a 128-byte
// zero patch instead); the staged rows are zero past K, so no bounds checks.
// poff: the lane's weight pieces within a block.
template <int W8>
__device__ __forceinline__ void slot_mma(float (&acc)[4][4], uint32_t st, int n, uint32_t xl, uint32_t cst, int c0,
                                         const int (&poff)[4]) {
    constexpr int BB = W8 ? kBlockBytesFp8 : kBlockBytesBf16;
    constexpr int CB = kStepChunk / BB;
#pragma unroll
    for (int b = 0; b < CB; b++) {
        if (b < n) {
            const uint32_t blk = st + b * BB;
            const uint32_t xk = xl + (uint32_t)(c0 + b) * cst;  // 64 k of bf16 / f16 (0: the zero lanes)
            float(&A0)[4] = acc[(b & 1) * 2];
            float(&A1)[4] = acc[(b & 1) * 2 + 1];
            if (!W8) {
                const uint4 w0 = lds128(blk + poff[0]), w1 = lds128(blk + poff[1]);
                const uint4 w2 = lds128(blk + poff[2]), w3 = lds128(blk + poff[3]);
                const uint4 x0 = lds128(xk), x1 = lds128(xk + 64);
                mma_bf16_16816(A0, w0.x, w2.x, w0.y, w2.y, x0.x, x0.y);
                mma_bf16_16816(A1, w1.x, w3.x, w1.y, w3.y, x1.x, x1.y);
                mma_bf16_16816(A0, w0.z, w2.z, w0.w, w2.w, x0.z, x0.w);
                mma_bf16_16816(A1, w1.z, w3.z, w1.w, w3.w, x1.z, x1.w);
            } else {
                const uint4 ra = lds128(blk + poff[0]), rb = lds128(blk + poff[1]);
                const uint4 xlo = lds128(xk), xhi = lds128(xk + 16);
                mma_f16_16816(A0, e4m3x2_to_f16x2(ra.x & 0xffffu), e4m3x2_to_f16x2(rb.x & 0xffffu),
                              e4m3x2_to_f16x2(ra.x >> 16), e4m3x2_to_f16x2(rb.x >> 16), xlo.x, xlo.y);
                mma_f16_16816(A1, e4m3x2_to_f16x2(ra.y & 0xffffu), e4m3x2_to_f16x2(rb.y & 0xffffu),
                              e4m3x2_to_f16x2(ra.y >> 16), e4m3x2_to_f16x2(rb.y >> 16), xlo.z, xlo.w);
                mma_f16_16816(A0, e4m3x2_to_f16x2(ra.z & 0xffffu), e4m3x2_to_f16x2(rb.z & 0xffffu),
                              e4m3x2_to_f16x2(ra.z >> 16), e4m3x2_to_f16x2(rb.z >> 16), xhi.x, xhi.y);
                mma_f16_16816(A1, e4m3x2_to_f16x2(ra.w & 0xffffu), e4m3x2_to_f16x2(rb.w & 0xffffu),
                              e4m3x2_to_f16x2(ra.w >> 16), e4m3x2_to_f16x2(rb.w >> 16), xhi.z, xhi.w);
            }
        }
    }
}

__device__ __forceinline__ void run_epilogue(int epi, const GemvArgs& a, int tile, const float (&acc)[4], int g,
                                             int q, float (&bv)[2], int (&bi)[2]) {
    switch (epi) {
        case EPI_QKV: gemv_epilogue<EPI_QKV>(a, tile, acc, g, q, bv, bi); break;
        case EPI_RESID: gemv_epilogue<EPI_RESID>(a, tile, acc, g, q, bv, bi); break;
        case EPI_SWIGLU: gemv_epilogue<EPI_SWIGLU>(a, tile, acc, g, q, bv, bi); break;
        case EPI_LOGITS: gemv_epilogue<EPI_LOGITS>(a, tile, acc, g, q, bv, bi); break;
        default: gemv_epilogue<EPI_F32>(a, tile, acc, g, q, bv, bi); break;
    }
}

// The CTA's sum over a tile is complete (in acc, on one warp).  Tile inside
// the CTA's range: run the epilogue.  Shared with other CTAs: the first of
// them (slot 0, whose range ENDS in the tile) is the reducer; the others
// (whose ranges start there, so they finish it first) publish their partial
// and bump the tile's counter with a release reduction.  The reducer waits
// (bounded) for the n - 1 partials, adds them in slot order
// (deterministic), runs the epilogue and resets the counter.
__device__ void finish_tile(const StepCtl& c, const StepPhase& P, int tile, float (&acc)[4], int cta, int C, int g,
                            int q, int lane, float (&bv)[2], int (&bi)[2]) {
    const GemvArgs& a = P.g;
    const long long kc = a.kc;
    const int Cp = phase_ctas(P.blocks, C);
    const int first = block_owner(tile * kc, P.blocks, Cp), last = block_owner((tile + 1) * kc - 1, P.blocks, Cp);
    if (first != last) {
        const int slot = cta - first, n = last - first + 1;
        float4* base = c.part + (size_t)tile * P.slots * 32;
        if (slot != 0) {
            base[slot * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
            __syncwarp();
            if (lane == 0) red_release_add(c.tile_cnt + tile, 1u);
            return;
        }
        if (lane == 0) {
            const unsigned long long t0 = globaltimer();
            while (ld_acquire_u32(c.tile_cnt + tile) < (unsigned)(n - 1)) {
                if (ld_volatile_i32(c.abort)) break;
                if (globaltimer() - t0 > kWaitNs) {
                    atomicExch(c.abort, 1);
                    atomicExch(c.err, RENG_E_TIMEOUT);
                    break;
                }
            }
            c.tile_cnt[tile] = 0u;
        }
        __syncwarp();
        float4 s = make_float4(acc[0], acc[1], acc[2], acc[3]);
        for (int i = 1; i < n; i++) {
            const float4 v = __ldcg(base + i * 32 + lane);
            s.x += v.x;
            s.y += v.y;
            s.z += v.z;
            s.w += v.w;
        }
        acc[0] = s.x;
        acc[1] = s.y;
        acc[2] = s.z;
        acc[3] = s.w;
    }
    if (a.w8) {
        const float s0 = __ldg(a.wscale + tile * kTileRows + g), s1 = __ldg(a.wscale + tile * kTileRows + g + 8);
        acc[0] *= s0;
        acc[1] *= s0;
        acc[2] *= s1;
        acc[3] *= s1;
    }
    run_epilogue(P.epi, a, tile, acc, g, q, bv, bi);
}

// x_res[m] = embed[id], row bookkeeping and the norm partials (decode rows).
__device__ void embed_phase(const EmbedArgs& e) {
    const int nv = e.hidden / 8;
    const int total = e.M * nv;
    const int stride = gridDim.x * blockDim.x;
    const int step = *e.step;
    for (int base = blockIdx.x * blockDim.x; base < total; base += stride) {
        const int t = base + threadIdx.x;
        float ss = 0.f;
        const bool live = t < total;
        const int m = live ? t / nv : 0, i = live ? t % nv : 0;
        if (live) {
            const int pos = e.pos[m];
            uint32_t id = e.ids_ring[(size_t)step * e.batch + m];
            if (id >= (uint32_t)e.vocab) {  // reported, never read out of range
                if (i == 0) atomicCAS(e.err, 0, RENG_E_INVAL);
                id = 0;
            }
            if (i == 0) {
                e.row_slot[m] = m;
                e.row_pos[m] = pos;
            }
            const uint4 v = ldg_nc(reinterpret_cast<const uint4*>(e.table + (size_t)id * e.hidden) + i);
            reinterpret_cast<uint4*>(e.x_res + (size_t)m * e.hidden)[i] = v;
            const float f[8] = {bf16lo(v.x), bf16hi(v.x), bf16lo(v.y), bf16hi(v.y),
                                bf16lo(v.z), bf16hi(v.z), bf16lo(v.w), bf16hi(v.w)};
#pragma unroll
            for (int k = 0; k < 8; k++) ss += f[k] * f[k];
        }
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);  // nv is even: lanes 2j, 2j+1 hold one 16-wide tile
        if (live && (i & 1) == 0) e.ss_out[(size_t)m * kSsStride + (i >> 1)] = ss;
    }
}

// Attention scratch of a CTA (in the x staging buffer).
constexpr int kAKP = 128 + 8;  // padded key row (bf16): conflict-free 16-byte reads

struct AttnSmem {
    uint16_t K[kStepAttnKeys * kAKP];
    uint16_t V[kStepAttnKeys * kAKP];
    float Q[kAttnMaxHpgStep * 128];
    float P[kAttnMaxHpgStep][kStepAttnKeys];
    float M[kAttnMaxHpgStep], L[kAttnMaxHpgStep], Al[kAttnMaxHpgStep];
    int last;
};

// Attention over the KV cache: a CTA per unit (row m, KV group, key range
// of 32-key tiles), f32 scores and online softmax per tile as the
// per-projection attention kernel computes them; each unit publishes its
// unnormalised output with its running max and sum, and the last unit of
// (m, group) to finish combines the units in order and writes bf16.
__device__ void attn_phase(const StepCtl& c, const AttnArgs& a, AttnSmem& s) {
    const int A = c.attn_units;
    const int hpg = a.hpg, hd = a.hd, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q_dim = a.n_kv * hpg * hd;
    const int part_len = step_attn_part_len(hpg, hd);
    const int per_head = hd / 4;
    const int ph = tid / per_head, pd = (tid % per_head) * 4;
    const bool owns = tid < hpg * per_head;
    const int vec_per_row = hd / 8;
    for (int u = blockIdx.x; u < a.M * a.n_kv * A; u += gridDim.x) {
        const int unit = u % A, mg = u / A, m = mg / a.n_kv, grp = mg % a.n_kv;
        const int pos = __ldcg(a.row_pos + m), slot = __ldcg(a.row_slot + m);
        const int nkeys = min(pos + 1, a.cap);
        const int ntile = (nkeys + kStepAttnKeys - 1) / kStepAttnKeys;
        const int U = min(ntile, A);
        if (unit >= U) continue;  // uniform over the CTA
        const int t0 = unit * ntile / U, t1 = (unit + 1) * ntile / U;
        const size_t cache_base = (((size_t)slot * a.n_kv + grp) * a.cap) * hd;
        __syncthreads();  // the previous unit's reads of the scratch are done
        const uint16_t* qrow = a.q + (size_t)m * q_dim + (size_t)grp * hpg * hd;
        for (int i = tid; i < hpg * hd; i += blockDim.x) s.Q[i] = bf16_bits_to_f32(__ldcg(qrow + i));
        if (tid < kAttnMaxHpgStep) {
            s.M[tid] = -INFINITY;
            s.L[tid] = 0.f;
        }
        float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
        for (int t = t0; t < t1; t++) {
            const int k0 = t * kStepAttnKeys, kn = min(kStepAttnKeys, nkeys - k0);
            __syncthreads();  // previous tile consumed (and Q, M, L ready on the first)
            {
                // K and V rows of the tile: every load in flight before the
                // shared-memory stores (2 x 32 keys x hd/8 vectors <= 4 per thread)
                constexpr int kPer = 2 * kStepAttnKeys * (128 / 8) / (kStepWarps * 32);
                const int nvec = kn * vec_per_row;
                uint4 r[kPer];
#pragma unroll
                for (int e = 0; e < kPer; e++) {
                    const int i = tid + e * kStepWarps * 32;
                    if (i < 2 * nvec) {
                        const int which = i / nvec, rr = i % nvec, jj = rr / vec_per_row, v = rr % vec_per_row;
                        const size_t off = cache_base + (size_t)(k0 + jj) * hd + v * 8;
                        r[e] = __ldcg(reinterpret_cast<const uint4*>((which ? a.vcache : a.kcache) + off));
                    }
                }
#pragma unroll
                for (int e = 0; e < kPer; e++) {
                    const int i = tid + e * kStepWarps * 32;
                    if (i < 2 * nvec) {
                        const int which = i / nvec, rr = i % nvec, jj = rr / vec_per_row, v = rr % vec_per_row;
                        *reinterpret_cast<uint4*>((which ? s.V : s.K) + jj * kAKP + v * 8) = r[e];
                    }
                }
            }
            __syncthreads();
            // scores: thread -> (head, key)
            if (tid < hpg * kStepAttnKeys) {
                const int h = tid / kStepAttnKeys, j = tid % kStepAttnKeys;
                float sc = -INFINITY;
                if (j < kn) {
                    float acc = 0.f;
                    const float* qh = s.Q + h * hd;
                    for (int d = 0; d < hd; d += 8) {
                        const uint4 kv = *reinterpret_cast<const uint4*>(s.K + j * kAKP + d);
                        acc += qh[d + 0] * bf16lo(kv.x) + qh[d + 1] * bf16hi(kv.x) + qh[d + 2] * bf16lo(kv.y) +
                               qh[d + 3] * bf16hi(kv.y) + qh[d + 4] * bf16lo(kv.z) + qh[d + 5] * bf16hi(kv.z) +
                               qh[d + 6] * bf16lo(kv.w) + qh[d + 7] * bf16hi(kv.w);
                    }
                    sc = acc;
                }
                s.P[h][j] = sc;
            }
            __syncthreads();
            // online-softmax statistics: warp h
            if (warp < hpg) {
                const int h = warp;
                const float sv = s.P[h][lane];
                const float mx = warp_max(sv);
                const float m_old = s.M[h], m_new = fmaxf(m_old, mx);
                const float pv = lane < kn ? expf(sv - m_new) : 0.f;
                s.P[h][lane] = pv;
                const float sum = warp_sum(pv);
                if (lane == 0) {
                    const float alpha = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
                    s.Al[h] = alpha;
                    s.L[h] = s.L[h] * alpha + sum;
                    s.M[h] = m_new;
                }
            }
            __syncthreads();
            if (owns) {
                const float al = s.Al[ph];
                acc0 *= al;
                acc1 *= al;
                acc2 *= al;
                acc3 *= al;
                for (int j = 0; j < kn; j++) {
                    const float p = s.P[ph][j];
                    const uint2 vv = *reinterpret_cast<const uint2*>(s.V + j * kAKP + pd);
                    acc0 += p * bf16lo(vv.x);
                    acc1 += p * bf16hi(vv.x);
                    acc2 += p * bf16lo(vv.y);
                    acc3 += p * bf16hi(vv.y);
                }
            }
        }
        // publish this unit: o (unnormalised), max, sum
        float* part = c.apart + (size_t)mg * A * part_len;
        float* mine = part + (size_t)unit * part_len;
        if (owns) *reinterpret_cast<float4*>(mine + ph * hd + pd) = make_float4(acc0, acc1, acc2, acc3);
        if (tid < hpg) {
            mine[hpg * hd + tid] = s.M[tid];
            mine[hpg * hd + hpg + tid] = s.L[tid];
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) s.last = atomicAdd(c.acnt + mg, 1u) == (unsigned)(U - 1);
        __syncthreads();
        if (!s.last) continue;
        __threadfence();
        if (owns) {
            float mx = -INFINITY;
            for (int v = 0; v < U; v++) mx = fmaxf(mx, __ldcg(part + (size_t)v * part_len + hpg * hd + ph));
            float n0 = 0.f, n1 = 0.f, n2 = 0.f, n3 = 0.f, den = 0.f;
            for (int v = 0; v < U; v++) {
                const float* pv = part + (size_t)v * part_len;
                const float mv = __ldcg(pv + hpg * hd + ph);
                const float w = mv == -INFINITY ? 0.f : expf(mv - mx);
                den += w * __ldcg(pv + hpg * hd + hpg + ph);
                const float4 o = __ldcg(reinterpret_cast<const float4*>(pv + ph * hd + pd));
                n0 += w * o.x;
                n1 += w * o.y;
                n2 += w * o.z;
                n3 += w * o.w;
            }
            uint16_t* out = a.out + (size_t)m * q_dim + ((size_t)grp * hpg + ph) * hd + pd;
            out[0] = f32_to_bf16_bits(n0 / den);
            out[1] = f32_to_bf16_bits(n1 / den);
            out[2] = f32_to_bf16_bits(n2 / den);
            out[3] = f32_to_bf16_bits(n3 / den);
        }
        if (tid == 0) c.acnt[mg] = 0u;
    }
}

__device__ __forceinline__ void copy_words(void* dst, const void* src, int bytes) {
    for (int i = threadIdx.x; i < bytes / 4; i += blockDim.x)
        reinterpret_cast<uint32_t*>(dst)[i] = __ldg(reinterpret_cast<const uint32_t*>(src) + i);
}

}  // namespace

size_t step_attn_smem_bytes() { return sizeof(AttnSmem); }

__global__ void __launch_bounds__(kStepWarps * 32, 1) k_step(StepCtl c) {
    extern __shared__ __align__(128) uint8_t smem_dyn[];
    __shared__ __align__(8) unsigned long long bars[kStepWarps * kStepMaxStages];
    __shared__ __align__(8) unsigned long long xbar;
    __shared__ __align__(16) StepPhase s_ph[2];  // this phase and the next (copied before the barrier)
    __shared__ float s_red[kStepWarps][kMaxRows];
    __shared__ float inv_s[kMaxRows];
    __shared__ int s_ids[kMaxRows];
    __shared__ int s_last;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const int C = gridDim.x, cta = blockIdx.x;
    const long long G = (long long)C * kStepWarps;
    const long long gw = (long long)cta * kStepWarps + warp;  // argmax partial slot
    const int S = c.stages;
    const uint32_t ring = (uint32_t)__cvta_generic_to_shared(smem_dyn) + warp * S * kStepChunk;
    uint8_t* xbuf = smem_dyn + kStepWarps * S * kStepChunk;
    uint16_t* xs = reinterpret_cast<uint16_t*>(xbuf);
    StepSeq* seq = reinterpret_cast<StepSeq*>(xbuf + ((c.xbytes + 127) & ~127));
    const int nph = c.nph;
    copy_words(seq, c.seq, nph * (int)sizeof(StepSeq));
    copy_words(&s_ph[0], c.ph, (int)sizeof(StepPhase));
    __syncthreads();
    const uint32_t bar0 = (uint32_t)__cvta_generic_to_shared(&bars[warp * kStepMaxStages]);
    const uint32_t xbar_a = (uint32_t)__cvta_generic_to_shared(&xbar);

    // ---- the weight stream: S chunks ahead of the consumer ----
    Cursor pc;  // producer cursor (lane 0)
    cursor_seek(seq, nph, pc, 0, cta, C, warp);
    bool failed = false;
    int issued = 0, waited = 0;
    auto issue = [&](int j) {  // lane 0: chunk j of the sequence into slot j % S
        if (pc.p >= nph || failed) return;
        const int n = cursor_chunk(pc);
        const uint32_t bytes = (uint32_t)(n * pc.bb);
        const uint32_t bar = bar0 + (j % S) * 8;
        mbar_expect_tx(bar, bytes);
        tma_load_1d(ring + (j % S) * kStepChunk, cursor_src(pc), bytes, bar);
        cursor_advance(seq, nph, pc, n, cta, C, warp);
        issued = j + 1;
    };
    if (threadIdx.x == 0) mbar_init(xbar_a, 1);
    if (lane == 0) {
        for (int s = 0; s < S; s++) mbar_init(bar0 + s * 8, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int j = 0; j < S; j++) issue(j);
    }
    __syncthreads();
    if (threadIdx.x == 0 && blockIdx.x == 0 && c.trace != nullptr) c.trace[0] = globaltimer();

    int j = 0;          // consumer: next chunk of the sequence
    int xphase = 0;     // parity of the x staging barrier
    float best_v[2] = {-INFINITY, -INFINITY};
    int best_i[2] = {0x7fffffff, 0x7fffffff};

    for (int p = 0; p < c.nph; p++) {
        const StepPhase& P = s_ph[p & 1];
        const int kind = P.kind;  // uniform
        if (kind == PH_EMBED) {
            embed_phase(P.em);
        } else if (kind == PH_ATTN) {
            attn_phase(c, P.at, *reinterpret_cast<AttnSmem*>(xbuf));
        } else {
            const GemvArgs& a = P.g;
            const int K = a.K, Kp = a.kc * 64, xstride = step_xstride(K), M = a.M;
            // stage this phase's x rows (written by earlier phases, other SMs)
            if (threadIdx.x == 0) {
                asm volatile("fence.proxy.async;" ::: "memory");
                mbar_expect_tx(xbar_a, (uint32_t)(M * K * 2));
                for (int m = 0; m < M; m++)
                    tma_load_1d((uint32_t)__cvta_generic_to_shared(xs + m * xstride), a.x + (size_t)m * a.ldx,
                                (uint32_t)(K * 2), xbar_a);
            }
            if (a.ss_in != nullptr) {
                // RMS partials of every row with all loads in flight at once
                float v[kMaxRows][2];
#pragma unroll
                for (int m = 0; m < kMaxRows; m++)
#pragma unroll
                    for (int r = 0; r < 2; r++) {
                        const int t = threadIdx.x + r * kStepWarps * 32;
                        v[m][r] = (m < M && t < a.ss_tiles) ? __ldcg(a.ss_in + (size_t)m * kSsStride + t) : 0.f;
                    }
                for (int t = threadIdx.x + 2 * kStepWarps * 32; t < a.ss_tiles; t += kStepWarps * 32)
                    for (int m = 0; m < M; m++) v[m][0] += __ldcg(a.ss_in + (size_t)m * kSsStride + t);
#pragma unroll
                for (int m = 0; m < kMaxRows; m++) {
                    const float sm = warp_sum(v[m][0] + v[m][1]);
                    if (lane == 0) s_red[warp][m] = sm;
                }
            }
            if (!mbar_wait_bounded(xbar_a, (uint32_t)(xphase & 1))) {
                if (threadIdx.x == 0) {
                    atomicExch(c.abort, 1);
                    atomicExch(c.err, RENG_E_TIMEOUT);
                }
            }
            xphase++;
            __syncthreads();
            if (a.ss_in != nullptr && threadIdx.x < M) {
                float sm = 0.f;
                for (int w = 0; w < kStepWarps; w++) sm += s_red[w][threadIdx.x];
                inv_s[threadIdx.x] = 1.0f / sqrtf(sm / (float)a.norm_k + a.eps);
            }
            __syncthreads();
            if (a.ss_in != nullptr) {
                if (a.w8) normalise_x<1>(a, xs, xstride, K, inv_s);
                else normalise_x<0>(a, xs, xstride, K, inv_s);
            } else if (a.w8) {
                x_to_f16(a, xs, xstride, K);
            }
            // zeros past K in every row and a 128-byte zero patch after the
            // rows (read by the lanes of rows >= M): no bounds checks
            for (int i = threadIdx.x; i < M * ((Kp - K) / 2) + 32; i += blockDim.x) {
                if (i < 32) {
                    reinterpret_cast<uint32_t*>(xs + M * xstride)[i] = 0u;
                } else {
                    const int r = i - 32, m = r / ((Kp - K) / 2), k = K + (r % ((Kp - K) / 2)) * 2;
                    *reinterpret_cast<uint32_t*>(xs + m * xstride + k) = 0u;
                }
            }
            __syncthreads();
            if (threadIdx.x == 0 && blockIdx.x == 0 && c.trace != nullptr) c.trace[kTraceStride * p + 3] = globaltimer();
            // the CTA's tiles: each warp streams its share of a tile, the
            // shares are added in shared memory (warp order), and one warp
            // (rotating) finishes the tile while the others go on
            const bool w8 = a.w8 != 0;
            const uint32_t xl = (uint32_t)__cvta_generic_to_shared(g < M ? xs + g * xstride + (w8 ? q * 16 : q * 8)
                                                                         : xs + M * xstride);
            const uint32_t cst = g < M ? 128u : 0u;
            int poff[4];
            if (w8) lane_pieces<1>(g, q, lane, poff);
            else lane_pieces<0>(g, q, lane, poff);
            const int qn = (M + 1) / 2;  // lanes q < qn hold the M columns
            float4* red = reinterpret_cast<float4*>(xbuf + ((M * xstride * 2 + 128 + 15) & ~15));
            const int kc = a.kc, bb = w8 ? kBlockBytesFp8 : kBlockBytesBf16;
            int lo, hi;
            cta_range(P.blocks, C, cta, lo, hi);
            const int t_first = lo / kc, t_last = lo < hi ? (hi - 1) / kc : t_first - 1;
            for (int t = t_first; t <= t_last; t++) {
                int s0, s1;
                warp_share(lo, hi, kc, t, warp, s0, s1);
                float acc4[4][4] = {};
                for (int pos = s0; pos < s1;) {
                    const int n = min(kStepChunk / bb, s1 - pos);
                    const uint32_t slot = ring + (j % S) * kStepChunk;
                    if (!failed) {
                        if (mbar_wait_bounded(bar0 + (j % S) * 8, (uint32_t)((j / S) & 1))) {
                            waited = j + 1;
                        } else {
                            failed = true;
                            if (lane == 0) {
                                atomicExch(c.abort, 1);
                                atomicExch(c.err, RENG_E_TIMEOUT);
                            }
                        }
                    }
                    if (w8) slot_mma<1>(acc4, slot, n, xl, cst, pos - t * kc, poff);
                    else slot_mma<0>(acc4, slot, n, xl, cst, pos - t * kc, poff);
                    __syncwarp();
                    if (lane == 0) {
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        issue(j + S);
                    }
                    __syncwarp();
                    j++;
                    pos += n;
                }
                if (q < qn)
                    red[(warp * 8 + g) * qn + q] =
                        make_float4((acc4[0][0] + acc4[1][0]) + (acc4[2][0] + acc4[3][0]),
                                    (acc4[0][1] + acc4[1][1]) + (acc4[2][1] + acc4[3][1]),
                                    (acc4[0][2] + acc4[1][2]) + (acc4[2][2] + acc4[3][2]),
                                    (acc4[0][3] + acc4[1][3]) + (acc4[2][3] + acc4[3][3]));
                __syncthreads();
                const bool mine = warp == t % kStepWarps;
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
                if (mine && q < qn) {
                    for (int w = 0; w < kStepWarps; w++) {
                        const float4 v = red[(w * 8 + g) * qn + q];
                        acc[0] += v.x;
                        acc[1] += v.y;
                        acc[2] += v.z;
                        acc[3] += v.w;
                    }
                }
                __syncthreads();
                if (mine) finish_tile(c, P, t, acc, cta, C, g, q, lane, best_v, best_i);
            }
            if (lane == 0 && blockIdx.x == 0 && c.trace != nullptr) atomicMax(c.trace + kTraceStride * p + 4, globaltimer());
            if (P.epi == EPI_LOGITS) {
                // this warp's best per row (lanes g == 0 hold rows 2q, 2q + 1)
                if (g == 0 && 2 * q < kMaxRows) {
                    c.am_val[gw * kMaxRows + 2 * q] = best_v[0];
                    c.am_idx[gw * kMaxRows + 2 * q] = best_i[0];
                    c.am_val[gw * kMaxRows + 2 * q + 1] = best_v[1];
                    c.am_idx[gw * kMaxRows + 2 * q + 1] = best_i[1];
                }
                __threadfence();
                __syncthreads();
                if (threadIdx.x == 0) s_last = atomicAdd(a.am_count, 1u) == gridDim.x - 1;
                __syncthreads();
                if (s_last) {
                    __threadfence();
                    for (int m = warp; m < M; m += kStepWarps) {
                        float bv = -INFINITY;
                        int bi = 0x7fffffff;
                        for (long long w = lane; w < G; w += 32)
                            am_take(bv, bi, __ldcg(c.am_val + w * kMaxRows + m), __ldcg(c.am_idx + w * kMaxRows + m));
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) {
                            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                            am_take(bv, bi, ov, oi);
                        }
                        if (lane == 0) s_ids[m] = bi == 0x7fffffff ? 0 : bi;  // all NaN: index 0
                    }
                    __syncthreads();
                    if (threadIdx.x == 0) {
                        const int s = *a.step;
                        for (int m = 0; m < M; m++) {
                            a.ids_ring[(size_t)(s + 1) * a.batch + m] = (uint32_t)s_ids[m];
                            a.pos[m] += 1;
                        }
                        *a.step = s + 1;
                        *a.am_count = 0u;
                        __threadfence();
                    }
                }
            }
        }
        if (p + 1 < c.nph) {
            // the next phase's arguments: loads in flight across the barrier
            copy_words(&s_ph[(p + 1) & 1], c.ph + p + 1, (int)sizeof(StepPhase));
            grid_sync(c, p);
        }
    }
    if (threadIdx.x == 0 && c.trace != nullptr) {  // the last phase has no barrier
        const unsigned long long t = globaltimer();
        atomicMin(c.trace + kTraceStride * (c.nph - 1) + 1, t);
        atomicMax(c.trace + kTraceStride * (c.nph - 1) + 2, t);
    }
    // drain this warp's own copies still in flight (only after a wait gave up)
    if (failed && lane == 0) {
        for (int jj = waited; jj < issued; jj++)
            if (!mbar_wait_bounded(bar0 + (jj % S) * 8, (uint32_t)((jj / S) & 1))) break;
    }
}

size_t step_smem_bytes(int stages, int xbytes, int nph) {
    return (size_t)kStepWarps * stages * kStepChunk + (size_t)((xbytes + 127) & ~127) +
           (size_t)nph * sizeof(StepSeq);
}

int step_blocks_per_sm(int /*w8*/, int stages, int xbytes, int nph) {
    const size_t smem = step_smem_bytes(stages, xbytes, nph);
    if (smem > 227 * 1024) return 0;
    if (cudaFuncSetAttribute(k_step, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_step, kStepWarps * 32, smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

cudaError_t launch_step(const StepCtl& c, int /*w8*/, int grid, cudaStream_t st) {
    if (c.stages < 1 || c.stages > kStepMaxStages) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kStepWarps * 32);
    cfg.dynamicSmemBytes = step_smem_bytes(c.stages, c.xbytes, c.nph);
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_step, c);
}

}  // namespace reng
