// Prefill-block attention on the tensor cores (a flash attention over the
// HBM-resident KV cache): the rows of a prefill block are consecutive
// positions of one slot, so a CTA takes a tile of them and walks the cache
// in 128-key tiles with an online softmax, never forming a score matrix.
//
// Tile: one KV group's hpg query heads x P = 128 / hpg positions are the
// 128 rows of the MMA (row r: head r / P, position r % P), so one K/V tile
// serves every head of the group.  Per 128-key tile:
//   S = Q K^T   tcgen05.mma kind::f16, M 128, N 128 keys, K = head_dim;
//               Q (K-major) staged by the softmax warps, K (K-major) by TMA
//               straight from the cache ([keys][head_dim] rows, 128-byte
//               swizzle), S in TMEM columns 0..127;
//   softmax     two threads own each TMEM lane (query row), one per half
//               of the 128 keys (warps w and w + 4 read the same lane
//               quarter): tcgen05.ld of the half's 64 scores, causal mask
//               (key <= the row's position), the row max swapped between
//               the halves through shared memory, running max and sum in
//               f32, P = exp(s - max) as bf16 into shared memory in the
//               K-major A-operand layout (each half one 64-key block), O
//               rescaled in TMEM (tcgen05.ld / st, each half its columns)
//               when the max moved;
//   O += P V    M 128, N = head_dim, K 128 keys; V read MN-major from the
//               same TMA layout (64-dim blocks 16 KB apart, 8-key groups
//               1 KB apart), O in TMEM columns 128..128+head_dim.
// Roles (320 threads): warp 0 lane 0 issues the K/V copies (two stages),
// warp 1 owns TMEM (256 columns) and lane 0 issues the MMAs, warps 2-9 stage
// Q, run the softmax and write O / l as bf16.  The softmax is the kernel's
// critical path (one exponential per score on the CUDA cores): two threads
// per row halve it, measured on B200 against one thread per row.  Every mbarrier wait is
// bounded; a wait that runs out records RENG_E_TIMEOUT and the kernel ends.
// The attention scale is already in q (folded into the bf16 wq), as the
// per-row kernel assumes (crates/reng-synapse/src/model.rs:151-157).
#include <mutex>
#include <string>

#include "gemm.cuh"
#include "tc.cuh"

namespace reng {
using namespace tc;

namespace {
constexpr int kFaThreads = 320;
constexpr int kFaRows = 128;     // query rows of a tile (the MMA's M)
constexpr int kFaKeys = 128;     // keys of a K/V tile
constexpr int kFaBlock = 16384;  // one 128-row x 128-byte swizzled operand block

struct FaArgs {
    const uint16_t* q;    // [M][q_dim], RoPE applied, attention scale folded in
    uint16_t* out;        // [M][q_dim]
    const int* row_slot;  // the block's slot (row 0)
    const int* row_pos;   // row 0's position; row m is at row_pos[0] + m
    int* err;
    int M, n_kv, hpg, hd, cap, P;
};

// Shared-memory address of 16-byte chunk `ch` of row r in a 128-byte-swizzled
// block (8-row atoms of 1024 B, chunk ch of row r at ch ^ (r % 8)).
__device__ __forceinline__ uint32_t swz(uint32_t block, int r, int ch) {
    return block + (uint32_t)(r >> 3) * 1024u + (uint32_t)(r & 7) * 128u + (uint32_t)((ch ^ (r & 7)) << 4);
}
// A bounded wait whose outcome every lane of the warp shares (the tcgen05
// loads and stores that follow are warp-collective).
__device__ __forceinline__ bool warp_wait(uint32_t b, uint32_t parity) {
    return __all_sync(0xffffffffu, bar_wait(b, parity));
}
// Named barrier 1 over the 256 softmax threads that also ANDs a flag across
// them: every thread leaves with the same answer, so a bounded wait that gave
// up in one warp ends the tile loop in all of them at the same barrier.
__device__ __forceinline__ bool softmax_all(bool v) {
    int r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.s32 p, %1, 0;\n\tbar.red.and.pred q, 1, 256, p;\n\t"
        "selp.s32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((int)v)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void st_shared16(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
}  // namespace

__global__ void __launch_bounds__(kFaThreads, 1) k_attn_prefill(const __grid_constant__ CUtensorMap kmap,
                                                                const __grid_constant__ CUtensorMap vmap, FaArgs f) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ __align__(8) unsigned long long kv_full[2], kv_empty[2], q_full, s_full, s_free, p_full, o_done, drain;
    __shared__ uint32_t tmem_base_s;
    __shared__ float xmax[2][2][kFaRows];  // [tile parity][half][row] the halves' row maxima
    __shared__ float xsum[2][kFaRows];     // [half][row] the halves' running sums at the end

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NC = f.hd >> 6;  // 64-wide head-dim blocks (1 or 2)
    const uint32_t smem0 = ((uint32_t)__cvta_generic_to_shared(smem_raw) + 1023u) & ~1023u;
    const uint32_t sQ = smem0, sK = sQ + (uint32_t)NC * kFaBlock, sV = sK + 2u * NC * kFaBlock,
                   sP = sV + 2u * NC * kFaBlock;
    auto bar = [](unsigned long long* b) { return (uint32_t)__cvta_generic_to_shared(b); };
    const int grp = blockIdx.y, t0 = blockIdx.x * f.P;

    if (threadIdx.x == 0) {
        for (int s = 0; s < 2; s++) {
            bar_init(bar(&kv_full[s]), 1);
            bar_init(bar(&kv_empty[s]), 1);
        }
        bar_init(bar(&q_full), 8);
        bar_init(bar(&s_full), 1);
        bar_init(bar(&s_free), 8);
        bar_init(bar(&p_full), 8);
        bar_init(bar(&o_done), 1);
        bar_init(bar(&drain), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        const uint32_t dst = (uint32_t)__cvta_generic_to_shared(&tmem_base_s);
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(dst) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_s, tS = tmem, tO = tmem + 128;

    // q and this block's keys and values come from the q/k/v launch
    pdl_wait();
    pdl_launch();
    const int pos0 = __ldcg(f.row_pos), slot = __ldcg(f.row_slot);
    const int last = min(f.M, t0 + f.P) - 1;
    const int ntiles = (pos0 + last + kFaKeys) / kFaKeys;  // keys 0 .. pos0 + last
    const long long ybase = ((long long)slot * f.n_kv + grp) * f.cap;

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            for (int j = 0; j < ntiles; j++) {
                const int s = j & 1;
                if (j >= 2 && !bar_wait(bar(&kv_empty[s]), (uint32_t)(((j >> 1) - 1) & 1))) {
                    atomicExch(f.err, RENG_E_TIMEOUT);
                    break;
                }
                bar_expect_tx(bar(&kv_full[s]), 2u * NC * kFaBlock);
                const int y = (int)(ybase + (long long)j * kFaKeys);
                for (int c = 0; c < NC; c++) {
                    tensor_g2s(sK + (uint32_t)(s * NC + c) * kFaBlock, &kmap, c * 64, y, bar(&kv_full[s]));
                    tensor_g2s(sV + (uint32_t)(s * NC + c) * kFaBlock, &vmap, c * 64, y, bar(&kv_full[s]));
                }
                issued = j + 1;
            }
            // the last copy into each stage has landed before the CTA may exit
            for (int j = max(0, issued - 2); j < issued; j++)
                if (!bar_wait(bar(&kv_full[j & 1]), (uint32_t)((j >> 1) & 1))) atomicExch(f.err, RENG_E_TIMEOUT);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idS = umma_idesc(kFaKeys);
            const uint32_t idO = umma_idesc(f.hd) | (1u << 16);  // B (V) MN-major
            bool ok = bar_wait(bar(&q_full), 0);
            for (int j = 0; j < ntiles && ok; j++) {
                const int s = j & 1;
                ok = bar_wait(bar(&kv_full[s]), (uint32_t)((j >> 1) & 1)) &&
                     (j == 0 || bar_wait(bar(&s_free), (uint32_t)((j - 1) & 1)));
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                for (int c = 0; c < NC; c++)
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        umma(tS, umma_desc(sQ + (uint32_t)c * kFaBlock + kk * 32),
                             umma_desc(sK + (uint32_t)(s * NC + c) * kFaBlock + kk * 32), idS, (c | kk) ? 1u : 0u);
                umma_commit(bar(&s_full));
                if (!(ok = bar_wait(bar(&p_full), (uint32_t)(j & 1)))) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t v0 = sV + (uint32_t)s * NC * kFaBlock;
                for (int h2 = 0; h2 < 2; h2++)
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        umma(tO, umma_desc(sP + (uint32_t)h2 * kFaBlock + kk * 32),
                             umma_desc_mn(v0 + (uint32_t)(h2 * 64 + kk * 16) * 128u, kFaBlock, 1024), idO,
                             (j | h2 | kk) ? 1u : 0u);
                umma_commit(bar(&o_done));
                umma_commit(bar(&kv_empty[s]));
            }
            if (!ok) atomicExch(f.err, RENG_E_TIMEOUT);
            // every MMA this thread issued has completed before TMEM is freed
            umma_commit(bar(&drain));
            if (!bar_wait(bar(&drain), 0)) atomicExch(f.err, RENG_E_TIMEOUT);
        }
    } else {
        // ---- warps 2..9: TMEM lane r = query row r of the tile, keys
        // 64 h .. 64 h + 63 of each key tile and O columns h hd/2 .. ----
        const int r = 32 * (warp & 3) + lane, h = (warp - 2) >> 2;
        const int hl = r / f.P, t = r % f.P, mrow = t0 + t;
        const bool active = hl < f.hpg && mrow < f.M;
        const int q_dim = f.n_kv * f.hpg * f.hd;
        const int head = grp * f.hpg + hl;
        const int pos = pos0 + mrow;
        const int ohalf = f.hd >> 1;  // O columns per half
        const uint32_t lanes = (uint32_t)(32 * (warp & 3)) << 16;
        {
            // Q row r: the half stages every other 16-byte chunk
            const uint4* qr = reinterpret_cast<const uint4*>(f.q + (size_t)mrow * q_dim + (size_t)head * f.hd);
            for (int c = 0; c < NC; c++)
#pragma unroll
                for (int ch = h; ch < 8; ch += 2)
                    st_shared16(swz(sQ + (uint32_t)c * kFaBlock, r, ch),
                                active ? __ldcg(qr + c * 8 + ch) : make_uint4(0u, 0u, 0u, 0u));
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) bar_arrive(bar(&q_full));
        float mrun = -INFINITY, lrun = 0.f;
        bool ok = true;
        for (int j = 0; j < ntiles; j++) {
            const bool okj = ok && warp_wait(bar(&s_full), (uint32_t)(j & 1));
            float sc[kFaKeys / 2];
            // causal: key j * 128 + 64 h + c is visible to this row iff it
            // is at or before the row's position
            const int lim = active ? pos - j * kFaKeys - h * (kFaKeys / 2) : -1;
            float mx = -INFINITY;
            if (okj) {
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
                for (int g = 0; g < kFaKeys / 32; g++) {
                    float v[16];
                    tmem_ld16(tS + lanes + h * (kFaKeys / 2) + g * 16, v);
#pragma unroll
                    for (int e = 0; e < 16; e++) sc[g * 16 + e] = v[e];
                }
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) bar_arrive(bar(&s_free));
#pragma unroll
                for (int c = 0; c < kFaKeys / 2; c++)
                    if (c <= lim) mx = fmaxf(mx, sc[c]);
            }
            // the row max over both halves (slots alternate by tile parity:
            // a slot is rewritten two tiles later, after the partner has
            // passed the next exchange, so after it read this one)
            xmax[j & 1][h][r] = mx;
            if (!softmax_all(okj)) {
                ok = false;
                break;
            }
            mx = fmaxf(mx, xmax[j & 1][h ^ 1][r]);
            const float mnew = fmaxf(mrun, mx);
            const float alpha = mrun == -INFINITY ? 0.f : __expf(mrun - mnew);
            float sum = 0.f;
#pragma unroll
            for (int c = 0; c < kFaKeys / 2; c++) {
                const float p = c <= lim ? __expf(sc[c] - mnew) : 0.f;
                sc[c] = p;
                sum += p;
            }
            lrun = lrun * alpha + sum;
            mrun = mnew;
            // P and O are free once the previous tile's P V has finished (a
            // wait that gives up ends the loop at the next exchange)
            if (j >= 1) {
                if (!warp_wait(bar(&o_done), (uint32_t)((j - 1) & 1))) {
                    ok = false;
                    continue;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            }
#pragma unroll
            for (int ch = 0; ch < 8; ch++) {
                const float* p = sc + ch * 8;
                st_shared16(swz(sP + (uint32_t)h * kFaBlock, r, ch),
                            make_uint4(pack_bf16x2(p[0], p[1]), pack_bf16x2(p[2], p[3]), pack_bf16x2(p[4], p[5]),
                                       pack_bf16x2(p[6], p[7])));
            }
            if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {
                for (int g = 0; g < ohalf / 16; g++) {
                    float v[16];
                    tmem_ld16(tO + lanes + h * ohalf + g * 16, v);
#pragma unroll
                    for (int e = 0; e < 16; e++) v[e] *= alpha;
                    tmem_st16(tO + lanes + h * ohalf + g * 16, v);
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) bar_arrive(bar(&p_full));
        }
        // the row's sum over both halves (every softmax thread takes this
        // barrier, also after a wait gave up, so none is left waiting)
        xsum[h][r] = lrun;
        asm volatile("bar.sync 1, 256;" ::: "memory");
        lrun += xsum[h ^ 1][r];
        if (ok && warp_wait(bar(&o_done), (uint32_t)((ntiles - 1) & 1))) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const float inv = lrun > 0.f ? 1.f / lrun : 0.f;
            uint4* dst = reinterpret_cast<uint4*>(f.out + (size_t)mrow * q_dim + (size_t)head * f.hd + h * ohalf);
            for (int g = 0; g < ohalf / 16; g++) {
                float v[16];
                tmem_ld16(tO + lanes + h * ohalf + g * 16, v);
                if (active) {
                    dst[2 * g] = make_uint4(pack_bf16x2(v[0] * inv, v[1] * inv), pack_bf16x2(v[2] * inv, v[3] * inv),
                                            pack_bf16x2(v[4] * inv, v[5] * inv), pack_bf16x2(v[6] * inv, v[7] * inv));
                    dst[2 * g + 1] =
                        make_uint4(pack_bf16x2(v[8] * inv, v[9] * inv), pack_bf16x2(v[10] * inv, v[11] * inv),
                                   pack_bf16x2(v[12] * inv, v[13] * inv), pack_bf16x2(v[14] * inv, v[15] * inv));
                }
            }
        } else {
            atomicExch(f.err, RENG_E_TIMEOUT);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem) : "memory");
    }
}

namespace {
size_t fa_smem_bytes(int hd) { return (size_t)(1 + 2 + 2) * (hd / 64) * kFaBlock + 2 * kFaBlock + 1024; }
}  // namespace

bool attn_prefill_fits(const AttnArgs& a, long long cache_rows) {
    return (a.hd == 64 || a.hd == 128) && a.hpg >= 1 && a.hpg <= kFaRows && a.contiguous &&
           cache_rows + kFaKeys < (1LL << 31);
}

int launch_attn_prefill(const AttnArgs& a, long long cache_rows, int* err, cudaStream_t st) {
    if (!attn_prefill_fits(a, cache_rows)) return fail(RENG_E_INVAL, "launch_attn_prefill: shape outside the kernel");
    static std::once_flag once;
    static cudaError_t prep = cudaSuccess;
    std::call_once(once, [] {
        prep = cudaFuncSetAttribute(k_attn_prefill, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)fa_smem_bytes(128));
    });
    if (prep != cudaSuccess) return fail(RENG_E_CUDA, std::string("attention prefill: ") + cudaGetErrorString(prep));
    CUtensorMap km, vm;
    int rc = attn_cache_map(a.kcache, a.hd, cache_rows, kFaKeys, &km);
    if (rc) return rc;
    rc = attn_cache_map(a.vcache, a.hd, cache_rows, kFaKeys, &vm);
    if (rc) return rc;
    FaArgs f{};
    f.q = a.q;
    f.out = a.out;
    f.row_slot = a.row_slot;
    f.row_pos = a.row_pos;
    f.err = err;
    f.M = a.M;
    f.n_kv = a.n_kv;
    f.hpg = a.hpg;
    f.hd = a.hd;
    f.cap = a.cap;
    f.P = kFaRows / a.hpg;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3((unsigned)((a.M + f.P - 1) / f.P), (unsigned)a.n_kv);
    cfg.blockDim = dim3(kFaThreads);
    cfg.dynamicSmemBytes = fa_smem_bytes(a.hd);
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_attn_prefill, km, vm, f);
    if (e != cudaSuccess) return fail(RENG_E_CUDA, std::string("attention prefill launch: ") + cudaGetErrorString(e));
    return RENG_OK;
}

}  // namespace reng
