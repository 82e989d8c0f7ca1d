// Decode attention over the HBM-resident KV cache with the key and value
// tiles streamed through a TMA ring (split-K flash decode, GQA).
//
// Grid and split as the per-row kernel (decode.cu, k_attn): one
// thread-block cluster of ns CTAs per (row, KV group), CTA s taking the s-th
// contiguous slice of the row's keys 0..pos, an f32 online softmax over
// 64-key tiles for all hpg query heads of the group at once, and the slices
// combined through distributed shared memory.  What changes is how a tile
// arrives: thread 0 issues one 2-D tensor-map copy per 64 head dims of K and
// of V (64 keys x 128 bytes, 128-byte swizzle) into a ring of stages, each
// with a bounded mbarrier wait, so the next tiles stream in while the CTA
// computes on this one; the per-row kernel loaded each tile with plain loads
// between two barriers.  Tiles whose keys were all written by earlier
// launches go out before the wait on the q/k/v kernel.  The reads of the
// swizzled rows (a key's row, or 4 dims of a row) are conflict-free.
#include <cooperative_groups.h>

#include <string>

#include "gemm.cuh"
#include "gemv_core.cuh"
#include "tc.cuh"

namespace reng {
using namespace tc;

namespace {
constexpr int kDaThreads = 256;
constexpr int kDaKeys = 64;           // keys per tile
constexpr int kDaMaxHpg = 8;
constexpr int kDaMaxHd = 128;
constexpr int kDaBox = kDaKeys * 128;  // one 64-key x 64-dim swizzled box (8 KB)
constexpr int kDaStages = 2;

// Byte offset of 16-byte chunk ch (dims 8 ch .. 8 ch + 7 of a 64-dim box) of
// key row j in a 128-byte-swizzled box.
__device__ __forceinline__ uint32_t da_swz(int j, int ch) {
    return (uint32_t)(j >> 3) * 1024u + (uint32_t)(j & 7) * 128u + (uint32_t)((ch ^ (j & 7)) << 4);
}
__device__ __forceinline__ uint2 lds64(uint32_t saddr) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(saddr));
    return v;
}
}  // namespace

__global__ void __launch_bounds__(kDaThreads) k_attn_ring(const __grid_constant__ CUtensorMap kmap,
                                                          const __grid_constant__ CUtensorMap vmap, AttnArgs a,
                                                          int* err) {
    namespace cg = cooperative_groups;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ __align__(16) float Qs[kDaMaxHpg * kDaMaxHd];
    __shared__ float Ps[kDaMaxHpg][kDaKeys];
    __shared__ float Ms[kDaMaxHpg], Ls[kDaMaxHpg], Al[kDaMaxHpg];
    __shared__ __align__(16) float Os[kDaMaxHpg * kDaMaxHd];  // this slice's unnormalised output
    __shared__ __align__(8) unsigned long long full[kDaStages];

    cg::cluster_group cluster = cg::this_cluster();
    const int s = (int)cluster.block_rank(), ns = (int)cluster.num_blocks();
    const int grp = blockIdx.y, m = blockIdx.z;
    const int hd = a.hd, hpg = a.hpg, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int NC = hd >> 6;  // 64-dim boxes per key row
    const uint32_t stage_bytes = 2u * (uint32_t)NC * kDaBox;
    const uint32_t smem0 = ((uint32_t)__cvta_generic_to_shared(smem_raw) + 1023u) & ~1023u;
    const uint32_t bar0 = (uint32_t)__cvta_generic_to_shared(&full[0]);
    // the row's position and slot were set by the step's embedding gather,
    // two launches back
    const int pos = __ldcg(a.row_pos + m);
    const int nkeys = min(pos + 1, a.cap);
    const int per = (nkeys + ns - 1) / ns;
    const int k0 = min(nkeys, s * per), k1 = min(nkeys, k0 + per);
    const int nt = (k1 - k0 + kDaKeys - 1) / kDaKeys;
    const int slot = __ldcg(a.row_slot + m);
    const long long ybase = ((long long)slot * a.n_kv + grp) * a.cap;
    const int old_end = pos - (a.contiguous ? m : 0);  // keys below were written by earlier launches
    const int q_dim = a.n_kv * hpg * hd;

    // tile t -> stage t % kDaStages: K boxes, then V boxes (thread 0 only)
    auto issue = [&](int t) {
        const uint32_t base = smem0 + (uint32_t)(t % kDaStages) * stage_bytes;
        const uint32_t b = bar0 + 8u * (uint32_t)(t % kDaStages);
        bar_expect_tx(b, stage_bytes);
        const int y = (int)(ybase + k0 + t * kDaKeys);
        for (int c = 0; c < NC; c++) {
            tensor_g2s(base + (uint32_t)c * kDaBox, &kmap, c * 64, y, b);
            tensor_g2s(base + (uint32_t)(NC + c) * kDaBox, &vmap, c * 64, y, b);
        }
    };
    if (tid == 0) {
        for (int st = 0; st < kDaStages; st++) bar_init(bar0 + 8u * st, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncthreads();
    int issued = 0;  // thread 0: tiles whose copies went out
    if (tid == 0) {
        // tiles wholly below the keys the q/k/v launch writes do not wait for it
        while (issued < min(kDaStages, nt) && k0 + (issued + 1) * kDaKeys <= old_end) issue(issued++);
    }
    pdl_wait();
    pdl_launch();
    if (tid == 0)
        while (issued < min(kDaStages, nt)) issue(issued++);

    const uint16_t* qrow = a.q + (size_t)m * q_dim + (size_t)grp * hpg * hd;
    for (int i = tid; i < hpg * hd; i += kDaThreads) Qs[i] = bf16_bits_to_f32(qrow[i]);
    if (tid < kDaMaxHpg) {
        Ms[tid] = -INFINITY;
        Ls[tid] = 0.f;
    }
    // PV ownership: thread -> (head, 4 output dims); hpg * hd / 4 <= 256
    const int per_head = hd / 4;
    const int ph = tid / per_head, pd = (tid % per_head) * 4;
    const bool owns = tid < hpg * per_head;
    float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
    __syncthreads();  // Qs, Ms, Ls

    int done = 0;  // tiles consumed
    for (int t = 0; t < nt; t++) {
        const int st = t % kDaStages;
        // every thread waits for the tile; a wait that gave up anywhere ends
        // the walk for the whole CTA (the slice's partial is then invalid,
        // and the error word says so), which still joins the cluster below
        const bool got = bar_wait(bar0 + 8u * st, (uint32_t)((t / kDaStages) & 1));
        if (!__syncthreads_and(got)) {
            if (tid == 0) atomicExch(err, RENG_E_TIMEOUT);
            break;
        }
        done = t + 1;
        const uint32_t kb = smem0 + (uint32_t)st * stage_bytes, vb = kb + (uint32_t)NC * kDaBox;
        const int c0 = k0 + t * kDaKeys, kn = min(kDaKeys, k1 - c0);
        // scores: thread -> key j, heads h = t/64, t/64 + 4, ...
        {
            const int j = tid & (kDaKeys - 1);
            for (int h = tid / kDaKeys; h < hpg; h += kDaThreads / kDaKeys) {
                float sc = -INFINITY;
                if (j < kn) {
                    float acc = 0.f;
                    const float* qh = Qs + h * hd;
                    for (int d = 0; d < hd; d += 8) {
                        const uint4 kv = lds128(kb + (uint32_t)(d >> 6) * kDaBox + da_swz(j, (d & 63) >> 3));
                        acc += qh[d + 0] * bf16lo(kv.x) + qh[d + 1] * bf16hi(kv.x) + qh[d + 2] * bf16lo(kv.y) +
                               qh[d + 3] * bf16hi(kv.y) + qh[d + 4] * bf16lo(kv.z) + qh[d + 5] * bf16hi(kv.z) +
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
            for (int j = lane; j < kDaKeys; j += 32) mx = fmaxf(mx, Ps[h][j]);
            mx = warp_max(mx);
            const float m_old = Ms[h], m_new = fmaxf(m_old, mx);
            float sum = 0.f;
            for (int j = lane; j < kDaKeys; j += 32) {
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
            const uint32_t vcol = vb + (uint32_t)(pd >> 6) * kDaBox;
            const int ch = (pd & 63) >> 3;
            const uint32_t sub = (uint32_t)(pd & 7) * 2u;
            for (int j = 0; j < kn; j++) {
                const float p = Ps[ph][j];
                const uint2 vv = lds64(vcol + da_swz(j, ch) + sub);
                acc0 += p * bf16lo(vv.x);
                acc1 += p * bf16hi(vv.x);
                acc2 += p * bf16lo(vv.y);
                acc3 += p * bf16hi(vv.y);
            }
        }
        __syncthreads();  // the stage is read: the async proxy may refill it
        if (tid == 0 && issued < nt) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(issued++);
        }
    }
    if (tid == 0) {
        // copies still in flight (a walk that ended early) land before the
        // CTA's shared memory goes away (bounded)
        for (int t = done; t < issued; t++)
            if (!bar_wait(bar0 + 8u * (t % kDaStages), (uint32_t)((t / kDaStages) & 1))) break;
    }
    if (owns) *reinterpret_cast<float4*>(&Os[ph * hd + pd]) = make_float4(acc0, acc1, acc2, acc3);
    cluster.sync();  // every slice's (Ms, Ls, Os) is complete and visible cluster-wide

    // combine: CTA s writes outputs o = s, s + ns, ... of the hpg * hd
    for (int o = s + ns * tid; o < hpg * hd; o += ns * kDaThreads) {
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

namespace {
size_t da_smem_bytes(int hd) { return (size_t)kDaStages * 2 * (hd / 64) * kDaBox + 1024; }
}  // namespace

bool attn_ring_fits(const AttnArgs& a, long long cache_rows) {
    return (a.hd == 64 || a.hd == 128) && a.hpg >= 1 && a.hpg <= kDaMaxHpg && a.hpg * (a.hd / 4) <= kDaThreads &&
           cache_rows + kDaKeys < (1LL << 31);
}

cudaError_t attn_ring_prepare() {
    return cudaFuncSetAttribute(k_attn_ring, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)da_smem_bytes(128));
}

int launch_attn_ring(const AttnArgs& a, long long cache_rows, int* err, bool pdl, cudaStream_t st) {
    if (!attn_ring_fits(a, cache_rows)) return fail(RENG_E_INVAL, "launch_attn_ring: shape outside the kernel");
    CUtensorMap km, vm;
    int rc = attn_cache_map(a.kcache, a.hd, cache_rows, kDaKeys, &km);
    if (rc) return rc;
    rc = attn_cache_map(a.vcache, a.hd, cache_rows, kDaKeys, &vm);
    if (rc) return rc;
    const int ns = attn_slices((long long)a.M * a.n_kv);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    cfg.gridDim = dim3(ns, a.n_kv, a.M);
    cfg.blockDim = dim3(kDaThreads);
    cfg.dynamicSmemBytes = da_smem_bytes(a.hd);
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = ns;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_attn_ring, km, vm, a, err);
    if (e != cudaSuccess) return fail(RENG_E_CUDA, std::string("decode attention launch: ") + cudaGetErrorString(e));
    return RENG_OK;
}

}  // namespace reng
