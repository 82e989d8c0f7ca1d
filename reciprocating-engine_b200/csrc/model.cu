// The decoder model behind the C ABI: weight upload and packing, the
// HBM-resident KV cache, the per-step kernel sequence, and the decode step
// captured once as a CUDA graph and replayed per token with the argmax fed
// back on the device (the reference's device decode loop,
// crates/reng-synapse/src/cached.rs:19-38, 752-835; batched.rs:1023-1151).
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <cstdlib>
#include <string>
#include <vector>

#include "gemm.cuh"

using namespace reng;

namespace reng {
int tp_init(reng_model* m, const uint8_t* id);
void tp_destroy(reng_model* m);
cudaError_t tp_allreduce(reng_model* m, float* buf, size_t count, cudaStream_t st);
cudaError_t launch_tp_residual(reng_model* m, const float* part, int M, bool pdl, cudaStream_t st);
cudaError_t launch_tp_ar_residual(reng_model* m, const float* part, int M, cudaStream_t st);
bool tp_p2p(reng_model* m, int M);
const HeadXchg* tp_head_xchg(reng_model* m);
int tp_exchange_kind(reng_model* m);
}  // namespace reng

struct LayerDev {
    uint8_t *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wd = nullptr;
    float *g1 = nullptr, *g2 = nullptr, *bqkv = nullptr;
    float *qn = nullptr, *kn = nullptr;  // q/k norm gains [hd] (qk_norm; qn carries the attention scale)
    bool no_rope = false;                // NoPE layer: the q/k/v launch rotates with the identity table
    // FP8 weights: per packed row scales (null for bf16)
    float *sqkv = nullptr, *so = nullptr, *sgu = nullptr, *sd = nullptr;
};

struct reng_model {
    reng_model_desc d{};
    int dev = 0;
    cudaStream_t st = nullptr;
    int sms = 148;
    // shape (local to this tensor-parallel rank)
    int hidden = 0, inter = 0, L = 0, nh = 0, nkv = 0, hd = 0, vocab = 0, B = 0, cap = 0;
    int q_dim = 0, kv_dim = 0, hpg = 0;
    int qkv_tiles = 0, q_tiles = 0, k_tiles = 0, o_tiles = 0, gu_tiles = 0, d_tiles = 0, lm_tiles = 0;
    std::vector<LayerDev> layers;
    uint8_t* lm = nullptr;
    uint16_t* embed = nullptr;
    float *final_gamma = nullptr, *rope_cos = nullptr, *rope_sin = nullptr;
    // q/k norm (Qwen3): the q/k/v launch rotates with the identity table and
    // k_qk_norm normalises and rotates with the real one
    bool qk_norm = false;
    bool any_no_rope = false;  // some layer rotates nothing (NoPE)
    float *rope_cos_id = nullptr, *rope_sin_id = nullptr;
    uint16_t *kcache = nullptr, *vcache = nullptr;
    size_t layer_kv = 0;  // elements per layer
    // work buffers
    uint16_t *x_res = nullptr, *qbuf = nullptr, *attn = nullptr, *act = nullptr, *logits = nullptr;
    uint16_t* xn = nullptr;          // RMS-normalised rows, the x operand of the tcgen05 GEMMs
    int launches = 0;                // kernels of this library enqueued so far
    bool gemv8 = true;               // 3..8-row projections on the register-fragment GEMV (RENG_GEMV8=0: off)
    float* gpart = nullptr;          // GEMM split-K partials (splits without a cluster)
    size_t gpart_floats = 0;
    int* gcnt = nullptr;             // GEMM split-K arrivals per super-tile
    float* ss = nullptr;
    float* part = nullptr;  // tensor-parallel f32 partials [kBlockRows][hidden]
    int *row_slot = nullptr, *row_pos = nullptr, *pos = nullptr, *step = nullptr;
    int* err = nullptr;  // device error word of the bounded waits
    int w8 = 0;          // projections held as FP8-E4M3 codes + row scales
    uint32_t *ids_ring = nullptr, *prefill_ids = nullptr, *next_id = nullptr;
    unsigned int* am_count = nullptr;
    unsigned long long* am_key = nullptr;  // [kBlockRows] LM-head argmax keys
    int lm_grid = 0;
    // GEMV launch shapes per kind (qkv, o, gate/up, down, LM head), for
    // M <= 2 and M > 2 activation rows
    int shape[5][2] = {};
    cudaGraphExec_t graph = nullptr;
    cudaGraphExec_t graph_full = nullptr;  // the step with the whole LM head (logits requests) when `graph` shards it
    int kernels_per_step = 0;
    std::vector<int> host_pos;
    uint32_t* pinned = nullptr;  // pinned staging: ids [kBlockRows], positions [kRowsCap], error word
    size_t bytes = 0;
    std::vector<void*> allocs;
    reng_step_times times{};
    // tensor parallel
    void* nccl = nullptr;
    int rank = 0, world = 1;
};

namespace {

// pinned staging words: a prefill block's ids [0, kBlockRows), the slots'
// positions, the device error word
constexpr int kPinnedPos = kBlockRows;
constexpr int kPinnedErr = kBlockRows + kRowsCap;
constexpr int kPinnedWords = kBlockRows + kRowsCap + 16;

template <typename T>
int dalloc(reng_model* m, T** p, size_t count) {
    size_t b = std::max<size_t>(count * sizeof(T), 16);
    cudaError_t e = cudaMalloc((void**)p, b);
    if (e != cudaSuccess)
        return fail(RENG_E_NOMEM, "cudaMalloc(" + std::to_string(b) + "): " + cudaGetErrorString(e));
    m->allocs.push_back(*p);
    m->bytes += b;
    return RENG_OK;
}

#define TRY(x)                  \
    do {                        \
        int rc__ = (x);         \
        if (rc__) return rc__;  \
    } while (0)

#define CU(x)                                                                               \
    do {                                                                                    \
        cudaError_t e__ = (x);                                                              \
        if (e__ != cudaSuccess)                                                             \
            return fail(RENG_E_CUDA, std::string(#x) + ": " + cudaGetErrorString(e__));     \
    } while (0)

// Copy `rows` x `cols` bf16 (source pitch `ld` elements) into `dst` (dense).
int copy_matrix(uint16_t* dst, const uint16_t* src, int64_t rows, int64_t cols, int64_t ld,
                int mem, cudaStream_t st) {
    cudaMemcpyKind k = mem == RENG_MEM_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
    if (ld == cols) {
        CU(cudaMemcpyAsync(dst, src, (size_t)rows * cols * 2, k, st));
    } else {
        CU(cudaMemcpy2DAsync(dst, (size_t)cols * 2, src, (size_t)ld * 2, (size_t)cols * 2, (size_t)rows, k, st));
    }
    return RENG_OK;
}

int pack(reng_model* m, uint8_t** out, const uint16_t* staged, const std::vector<int>& rowmap,
         int K, float scale, int scale_rows, int* tiles_out) {
    const int tiles = (int)(rowmap.size() / kTileRows);
    const int kc = (K + kChunkK - 1) / kChunkK;
    TRY(dalloc(m, out, (size_t)tiles * kc * kBlockBytesBf16));
    int* dmap = nullptr;
    CU(cudaMallocAsync((void**)&dmap, rowmap.size() * sizeof(int), m->st));
    CU(cudaMemcpyAsync(dmap, rowmap.data(), rowmap.size() * sizeof(int), cudaMemcpyHostToDevice, m->st));
    PackArgs a{};
    a.src = staged;
    a.ld = K;
    a.rowmap = dmap;
    a.tiles = tiles;
    a.K = K;
    a.kc = kc;
    a.scale = scale;
    a.scale_rows = scale_rows;
    a.dst = *out;
    CU(launch_pack(a, m->st));
    CU(cudaFreeAsync(dmap, m->st));
    CU(cudaStreamSynchronize(m->st));  // rowmap lives on the host stack
    if (tiles_out) *tiles_out = tiles;
    return RENG_OK;
}

// Quantize a staged bf16 matrix [src_rows][K] on the device (E4M3,
// per-channel absmax scales, backoff 1.0: reng_fp8::quantize_with's
// per-channel scheme) and pack the codes; the scales go to packed row order,
// the rows below scale_rows multiplied by `scale` (the attention scale on the
// q rows, which the bf16 path folds into wq).
int pack_fp8(reng_model* m, uint8_t** out, float** out_scales, const uint16_t* staged, int src_rows,
             const std::vector<int>& rowmap, int K, float scale, int scale_rows, int* tiles_out) {
    const int tiles = (int)(rowmap.size() / kTileRows);
    const int kc = (K + kChunkK - 1) / kChunkK;
    TRY(dalloc(m, out, (size_t)tiles * kc * kBlockBytesFp8));
    TRY(dalloc(m, out_scales, (size_t)tiles * kTileRows));
    uint8_t* codes = nullptr;
    float* sc = nullptr;
    int* dmap = nullptr;
    CU(cudaMallocAsync((void**)&codes, (size_t)src_rows * K, m->st));
    CU(cudaMallocAsync((void**)&sc, (size_t)src_rows * 4, m->st));
    CU(cudaMallocAsync((void**)&dmap, rowmap.size() * sizeof(int), m->st));
    CU(cudaMemcpyAsync(dmap, rowmap.data(), rowmap.size() * sizeof(int), cudaMemcpyHostToDevice, m->st));
    TRY(fp8_quantize_device(staged, src_rows, K, RENG_FP8_E4M3, RENG_SCALING_PCS, 1.0f, codes, sc, nullptr, m->st));
    Pack8Args a{};
    a.src = codes;
    a.rowmap = dmap;
    a.tiles = tiles;
    a.K = K;
    a.kc = kc;
    a.dst = *out;
    CU(launch_pack8(a, m->st));
    CU(launch_gather_scales(sc, dmap, tiles * kTileRows, scale, scale_rows, *out_scales, m->st));
    CU(cudaFreeAsync(codes, m->st));
    CU(cudaFreeAsync(sc, m->st));
    CU(cudaFreeAsync(dmap, m->st));
    CU(cudaStreamSynchronize(m->st));
    if (tiles_out) *tiles_out = tiles;
    return RENG_OK;
}

std::vector<int> plain_map(int rows) {
    int tiles = (rows + kTileRows - 1) / kTileRows;
    std::vector<int> v((size_t)tiles * kTileRows, -1);
    for (int r = 0; r < rows; r++) v[r] = r;
    return v;
}

__global__ void k_fill_f32(float* p, size_t n, float v) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        p[i] = v;
}

int upload_f32(reng_model* m, float** out, const float* src, size_t n, int mem) {
    TRY(dalloc(m, out, n));
    if (src == nullptr) {
        CU(cudaMemsetAsync(*out, 0, n * 4, m->st));
        return RENG_OK;
    }
    CU(cudaMemcpyAsync(*out, src, n * 4,
                       mem == RENG_MEM_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice, m->st));
    return RENG_OK;
}

// Launch shape of a GEMV kind (0 qkv, 1 o_proj, 2 gate/up, 3 down, 4 LM
// head) for few (M <= 2) and many activation rows: warps per CTA (4 or 8)
// + 100 (the TMA weight ring).  Measured on B200 (Llama-8B widths, whole
// decode step in its CUDA graph): 4-warp ring CTAs for every kind, 3.36 ms
// per step, against 3.91 ms with o_proj/down on 8-warp CTAs that streamed
// through registers (as fast alone, but their registers kept the next
// kernel's CTAs from starting early).
// RENG_GEMV_SHAPES="qkv,o,gu,down,lm" overrides both (a tuning knob).
void pick_shape(reng_model* m, int kind, int kc, int* shape_small, int* shape_big) {
    static const int small[5] = {104, 104, 104, 104, 104};
    static const int big[5] = {108, 108, 108, 108, 108};
    int ss = small[kind], sb = big[kind];
    if (kc < 32) ss = sb = 104;  // short K: 8 warps would leave warps without blocks
    const char* v = getenv("RENG_GEMV_SHAPES");
    if (v) {
        int vals[5] = {0, 0, 0, 0, 0}, n = 0;
        const char* p = v;
        while (*p && n < 5) {
            vals[n++] = atoi(p);
            while (*p && *p != ',') p++;
            if (*p == ',') p++;
        }
        const int x = kind < n ? vals[kind] : 0;
        if (x == 104 || x == 108) ss = sb = x;
    }
    *shape_small = ss;
    *shape_big = sb;
}

int validate(const reng_model_desc* d) {
    RENG_CHECK_ARG(d != nullptr, "reng_model_create: desc is NULL");
    RENG_CHECK_ARG(d->hidden > 0 && d->inter > 0 && d->n_layers > 0 && d->n_heads > 0 &&
                       d->n_kv_heads > 0 && d->head_dim > 0 && d->vocab > 0,
                   "reng_model_create: every dimension must be positive");
    RENG_CHECK_ARG(d->batch >= 1 && d->capacity >= 1, "reng_model_create: batch and capacity must be >= 1");
    RENG_CHECK_ARG(d->tp_world >= 1 && d->tp_rank >= 0 && d->tp_rank < d->tp_world,
                   "reng_model_create: bad tensor-parallel rank/world");
    RENG_CHECK_ARG(d->n_heads % d->n_kv_heads == 0, "reng_model_create: n_heads % n_kv_heads != 0");
    RENG_CHECK_ARG(d->n_heads % d->tp_world == 0 && d->n_kv_heads % d->tp_world == 0 &&
                       d->inter % d->tp_world == 0,
                   "reng_model_create: heads " + std::to_string(d->n_heads) + " / kv heads " +
                       std::to_string(d->n_kv_heads) + " / intermediate " + std::to_string(d->inter) +
                       " are not divisible by " + std::to_string(d->tp_world));
    RENG_CHECK_ARG(d->hidden % 16 == 0, "reng_model_create: hidden must be a multiple of 16");
    if (d->hidden > 16 * kSsStride)
        return fail(RENG_E_UNSUPPORTED, "reng_model_create: hidden above " + std::to_string(16 * kSsStride));
    RENG_CHECK_ARG(d->head_dim % 16 == 0 && d->head_dim <= 128,
                   "reng_model_create: head_dim must be a multiple of 16 and <= 128");
    RENG_CHECK_ARG(d->n_heads / d->n_kv_heads <= 8, "reng_model_create: more than 8 query heads per KV head");
    RENG_CHECK_ARG((d->inter / d->tp_world) % 8 == 0, "reng_model_create: intermediate per rank must be a multiple of 8");
    RENG_CHECK_ARG(d->weights == RENG_WEIGHTS_BF16 || d->weights == RENG_WEIGHTS_FP8_E4M3,
                   "reng_model_create: unknown weight format");
    RENG_CHECK_ARG(std::isfinite(d->eps) && d->eps >= 0.f && std::isfinite(d->attn_scale),
                   "reng_model_create: eps / attn_scale not finite");
    RENG_CHECK_ARG(d->capacity <= (1 << 20), "reng_model_create: capacity above 1048576 positions");
    // the FP8 GEMV reads x 16 columns at a time: every K it sees (hidden,
    // q width, intermediate per rank) must be a multiple of 16
    if (d->weights == RENG_WEIGHTS_FP8_E4M3 && (d->inter / d->tp_world) % 16 != 0)
        return fail(RENG_E_UNSUPPORTED, "reng_model_create: FP8 weights need the intermediate size per rank (" +
                                            std::to_string(d->inter / d->tp_world) + ") to be a multiple of 16");
    RENG_CHECK_ARG(d->qk_norm == 0 || d->qk_norm == 1, "reng_model_create: qk_norm must be 0 or 1");
    if (d->batch > kRowsCap)
        return fail(RENG_E_UNSUPPORTED, "reng_model_create: batch " + std::to_string(d->batch) + " above " +
                                            std::to_string(kRowsCap));
    return RENG_OK;
}

// Launch helpers, one per kernel of the step (all on stream `st`).
EmbedArgs embed_args(reng_model* m, int mode, int M, int slot) {
    EmbedArgs e{};
    e.table = m->embed;
    e.hidden = m->hidden;
    e.vocab = m->vocab;
    e.x_res = m->x_res;
    e.ss_out = m->ss;
    e.row_slot = m->row_slot;
    e.row_pos = m->row_pos;
    e.mode = mode;
    e.M = M;
    e.pos = m->pos;
    e.step = m->step;
    e.ids_ring = m->ids_ring;
    e.prefill_ids = m->prefill_ids;
    e.slot = slot;
    e.batch = m->B;
    e.err = m->err;
    return e;
}

int k_embed_launch(reng_model* m, int mode, int M, int slot, cudaStream_t st) {
    CU(launch_embed(embed_args(m, mode, M, slot), true, st));
    m->launches++;
    return RENG_OK;
}

GemvArgs base_args(reng_model* m) {
    GemvArgs g{};
    g.err = m->err;
    return g;
}

// k-chunks of a K-wide projection (64 k per packed block in both formats)
int proj_kc(reng_model* m, int K) {
    (void)m;
    return (K + kChunkK - 1) / kChunkK;
}

GemvArgs norm_args(reng_model* m, int M, const float* gain) {
    GemvArgs g = base_args(m);
    g.M = M;
    g.row_slot = m->row_slot;
    g.row_pos = m->row_pos;
    g.eps = m->d.eps;
    g.K = m->hidden;
    g.kc = (m->hidden + kChunkK - 1) / kChunkK;
    g.x = m->x_res;
    g.ldx = m->hidden;
    g.ss_in = m->ss;
    g.ss_tiles = m->hidden / kTileRows;
    g.gain = gain;
    g.norm_k = m->hidden;
    return g;
}

// Rows of a step above which projections run on the tcgen05 GEMM (bf16
// weights); at or below it the GEMV kernels (mma N = kMaxRows) stream the
// weights with the rows in registers.
// From 4 rows on, down_proj (kind 3) also runs on the GEMM: its GEMV would
// stage 4-8 rows of a wide x (inter = 14336), leaving the weight ring short
// (measured at batch 8: down 52 -> 30 us on the GEMM with plain K splits).
// The LM head (kind 4) does too unless the register-fragment GEMV takes it
// (173 against 206 us at batch 8).
bool use_gemm(const reng_model* m, int M, int kind) {
    if (m->w8) return M > kMaxRows;  // FP8: the GEMV up to its 8 rows, then the GEMM (codes converted in shared memory)
    return M > kMaxRows || (M >= 4 && (kind == 3 || (kind == 4 && !m->gemv8)));
}

// One projection: the GEMV for few rows, else (RMSNorm of x into xn when the
// projection normalises its input) the tcgen05 GEMM over N = M rounded up
// to 16 columns, in N-tiles of kRowsCap columns beyond that (prefill blocks
// of up to kBlockRows rows).  kind indexes the GEMV launch shapes.
int linear(reng_model* m, const GemvArgs& g, int epi, int kind, int max_grid, cudaStream_t st) {
    if (!use_gemm(m, g.M, kind)) {
        if (m->gemv8 && gemv8_fits(g)) {
            CU(launch_gemv8(g, epi, true, st));
        } else {
            CU(launch_gemv(g, epi, m->shape[kind][g.M > 2], max_grid, true, st));
        }
        m->launches++;
        return RENG_OK;
    }
    const uint16_t* x = g.x;
    if (g.ss_in != nullptr) {
        CU(launch_rmsnorm_rows(g.x, g.ss_in, g.ss_tiles, g.gain, g.eps, g.norm_k, m->xn, g.M, true, st));
        m->launches++;
        x = m->xn;
    }
    const int N = g.M > kRowsCap ? kRowsCap : (g.M + 15) / 16 * 16;
    GemmArgs a{};
    a.e = g;
    a.w = g.w;
    a.tiles16 = g.tiles;
    a.kc = g.kc;
    a.super_tiles = (g.tiles + 7) / 8;
    a.N = N;
    a.ntiles = (g.M + N - 1) / N;
    bool gsplit = false;
    gemm_plan(a.super_tiles * a.ntiles, g.kc, N, epi, m->sms, true, &a.ks, &a.stages, &gsplit, &a.C, g.w8 != 0);
    if (gsplit) {
        if ((size_t)a.super_tiles * a.ntiles * a.ks * 128 * N > m->gpart_floats ||
            a.super_tiles * a.ntiles > kGemmCntMax)
            return fail(RENG_E_STATE, "GEMM split-K scratch too small");
        a.gpart = m->gpart;
        a.gcnt = m->gcnt;
    }
    if (epi == EPI_LOGITS && (size_t)a.super_tiles > (size_t)m->lm_grid)
        return fail(RENG_E_STATE, "LM head argmax partials too small");
    a.b3d = g.K % kChunkK == 0;
    CUtensorMap map, wmap;
    if (a.b3d)
        TRY(gemm_tensor_map3(x, kBlockRows, g.K, N, a.C, &map));
    else
        TRY(gemm_tensor_map(x, kBlockRows, g.K, N, &map));
    if (g.w8)
        TRY(gemm_weight_map8(g.w, g.tiles, g.kc, a.C, &wmap));
    else
        TRY(gemm_weight_map(g.w, g.tiles, g.kc, a.C, &wmap));
    CU(launch_gemm_tc(map, wmap, a, epi, true, st));
    m->launches++;
    return RENG_OK;
}

GemvArgs qkv_args(reng_model* m, int l, int M) {
    const LayerDev& w = m->layers[l];
    GemvArgs g = norm_args(m, M, w.g1);
    g.w = w.wqkv;
    g.w8 = m->w8;
    g.wscale = w.sqkv;
    g.kc = proj_kc(m, m->hidden);
    g.tiles = m->qkv_tiles;
    g.out = m->qbuf;
    g.ldo = m->q_dim;
    g.bias = w.bqkv;
    g.head_dim = m->hd;
    g.q_tiles = m->q_tiles;
    g.k_tiles = m->k_tiles;
    g.n_kv = m->nkv;
    // q/k norm: raw q/k, rotated after the norm; NoPE: never rotated
    const bool id = m->qk_norm || w.no_rope;
    g.rope_cos = id ? m->rope_cos_id : m->rope_cos;
    g.rope_sin = id ? m->rope_sin_id : m->rope_sin;
    g.kcache = m->kcache + (size_t)l * m->layer_kv;
    g.vcache = m->vcache + (size_t)l * m->layer_kv;
    g.cap = m->cap;
    return g;
}

int k_qkv_launch(reng_model* m, int l, int M, cudaStream_t st) {
    TRY(linear(m, qkv_args(m, l, M), EPI_QKV, 0, 0, st));
    if (m->qk_norm) {  // per-head RMSNorm of q and k, then RoPE (model.rs:2962-3010)
        QkNormArgs a{};
        a.q = m->qbuf;
        a.kcache = m->kcache + (size_t)l * m->layer_kv;
        a.qn = m->layers[l].qn;
        a.kn = m->layers[l].kn;
        a.rope_cos = m->layers[l].no_rope ? m->rope_cos_id : m->rope_cos;
        a.rope_sin = m->layers[l].no_rope ? m->rope_sin_id : m->rope_sin;
        a.row_slot = m->row_slot;
        a.row_pos = m->row_pos;
        a.M = M;
        a.nq = m->nh;
        a.n_kv = m->nkv;
        a.hd = m->hd;
        a.cap = m->cap;
        a.q_dim = m->q_dim;
        a.eps = m->d.eps;
        CU(launch_qk_norm(a, true, st));
        m->launches++;
    }
    return RENG_OK;
}

AttnArgs attn_args(reng_model* m, int l, int M, int mode) {
    AttnArgs at{};
    at.contiguous = mode == 1;
    at.q = m->qbuf;
    at.kcache = m->kcache + (size_t)l * m->layer_kv;
    at.vcache = m->vcache + (size_t)l * m->layer_kv;
    at.out = m->attn;
    at.row_slot = m->row_slot;
    at.row_pos = m->row_pos;
    at.M = M;
    at.n_kv = m->nkv;
    at.hpg = m->hpg;
    at.hd = m->hd;
    at.cap = m->cap;
    return at;
}

// Attention of a step.  Prefill blocks of 16 or more rows run the
// tensor-core flash attention (attn_prefill.cu).  Decode steps and short
// blocks run the TMA-ring kernel (attn_decode.cu) in engines of at least
// kRingMinCap positions and the per-row kernel below that: measured on B200,
// the ring took Qwen2.5-32B b1 attention at 4096 cached positions from 55.3
// to 39.2 us per layer, but at short contexts its full 64-key tiles and its
// shared memory (half the CTAs per SM) lost (Llama-8B b1 at ~200 positions
// 6.1 -> 7.1 us, b64 22.8 -> 28.8 us).  The decode step is one captured
// graph, so the choice is the engine's, by its capacity (2048 keeps the
// engines sized for 1024-token prompts, as the bench's, on the per-row
// kernel: its b64 decode lost 10.5k -> 10.0k tok/s on the ring).
// RENG_FLASH_PREFILL=0 keeps every block on the per-row kernel and
// RENG_ATTN_RING=0 / 1 forces the decode choice (A/B knobs).
constexpr int kRingMinCap = 2048;
int k_attn_launch(reng_model* m, int l, int M, int mode, cudaStream_t st) {
    const AttnArgs a = attn_args(m, l, M, mode);
    const long long rows = (long long)m->B * m->nkv * m->cap;
    const char* env = getenv("RENG_FLASH_PREFILL");
    const char* rv = getenv("RENG_ATTN_RING");
    const bool ring = rv ? atoi(rv) != 0 : m->cap >= kRingMinCap;
    if (mode == 1 && M >= 16 && !(env && atoi(env) == 0) && attn_prefill_fits(a, rows)) {
        TRY(launch_attn_prefill(a, rows, m->err, st));
    } else if (ring && attn_ring_fits(a, rows)) {
        TRY(launch_attn_ring(a, rows, m->err, true, st));
    } else {
        CU(launch_attn(a, kAttnChunk, true, st));
    }
    m->launches++;
    return RENG_OK;
}

// o_proj (which == 0) or down_proj (which == 1) with the residual add; under
// tensor parallelism the f32 partial, the all-reduce and the residual kernel.
GemvArgs proj_args(reng_model* m, int l, int M, int which) {
    const LayerDev& w = m->layers[l];
    GemvArgs o = base_args(m);
    o.M = M;
    o.w = which == 0 ? w.wo : w.wd;
    o.tiles = which == 0 ? m->o_tiles : m->d_tiles;
    o.K = which == 0 ? m->q_dim : m->inter;
    o.kc = proj_kc(m, o.K);
    o.w8 = m->w8;
    o.wscale = which == 0 ? w.so : w.sd;
    o.x = which == 0 ? m->attn : m->act;
    o.ldx = o.K;
    o.out = m->x_res;
    o.ldo = m->hidden;
    o.ss_out = m->ss;
    o.out_f32 = m->part;
    return o;
}

int k_proj_launch(reng_model* m, int l, int M, int which, cudaStream_t st) {
    const GemvArgs o = proj_args(m, l, M, which);
    const int kind = which == 0 ? 1 : 3;
    if (m->world > 1) {
        TRY(linear(m, o, EPI_F32, kind, 0, st));
        if (tp_p2p(m, M)) {  // decode: one-shot peer all-reduce fused with the residual
            CU(launch_tp_ar_residual(m, m->part, M, st));
        } else {
            CU(tp_allreduce(m, m->part, (size_t)M * m->hidden, st));
            CU(launch_tp_residual(m, m->part, M, false, st));
        }
        m->launches++;
    } else {
        TRY(linear(m, o, EPI_RESID, kind, 0, st));
    }
    return RENG_OK;
}

GemvArgs gateup_args(reng_model* m, int l, int M) {
    const LayerDev& w = m->layers[l];
    GemvArgs u = norm_args(m, M, w.g2);
    u.w = w.wgu;
    u.w8 = m->w8;
    u.wscale = w.sgu;
    u.kc = proj_kc(m, m->hidden);
    u.tiles = m->gu_tiles;
    u.out = m->act;
    u.ldo = m->inter;
    return u;
}

int k_gateup_launch(reng_model* m, int l, int M, cudaStream_t st) {
    return linear(m, gateup_args(m, l, M), EPI_SWIGLU, 2, 0, st);
}

// LM head over rows [r0, r0 + M) of the step (logits and argmax rows 0..M-1).
// shard: this rank's vocabulary tiles only, the argmax keys exchanged with
// the other ranks (tensor-parallel decode; the logits of other ranks' rows
// are not written).
GemvArgs head_args(reng_model* m, int mode, int M, int slot, int r0, bool shard = false) {
    GemvArgs h = norm_args(m, M, m->final_gamma);
    h.x = m->x_res + (size_t)r0 * m->hidden;
    h.ss_in = m->ss + (size_t)r0 * kSsStride;
    h.w = m->lm;
    h.tiles = m->lm_tiles;
    if (shard) {
        const int t0 = (int)((long long)m->rank * m->lm_tiles / m->world);
        const int t1 = (int)((long long)(m->rank + 1) * m->lm_tiles / m->world);
        h.w = m->lm + (size_t)t0 * proj_kc(m, m->hidden) * kBlockBytesBf16;
        h.tiles = t1 - t0;
        h.row0 = t0 * kTileRows;
        h.hx = tp_head_xchg(m);
    }
    h.out = m->logits;
    h.ldo = m->vocab;
    h.vocab = m->vocab;
    h.am_count = m->am_count;
    h.am_key = m->am_key;
    h.mode = mode;
    h.slot = slot;
    h.batch = m->B;
    h.pos = m->pos;
    h.step = m->step;
    h.ids_ring = m->ids_ring;
    h.next_id = m->next_id;
    return h;
}

int k_head_launch(reng_model* m, int mode, int M, int slot, cudaStream_t st, int r0 = 0, bool shard = false) {
    return linear(m, head_args(m, mode, M, slot, r0, shard), EPI_LOGITS, 4, m->lm_grid, st);
}

// Whether decode steps shard the LM head over the tensor-parallel ranks:
// with the peer exchange set up and at most kMaxRows slots.
bool head_sharded(reng_model* m) {
    return m->world > 1 && m->B <= kMaxRows && tp_head_xchg(m) != nullptr;
}

// The kernels of one step.  mode 0: decode over the B slots (rows = slots,
// ids from the device ring).  mode 1: prefill of `M` ids of slot `slot`
// starting at the device position of that slot.  head: HEAD_NONE, HEAD_LAST
// (the LM head on the last row only: its logits land in row 0) or HEAD_ALL.
enum { HEAD_NONE = 0, HEAD_LAST = 1, HEAD_ALL = 2, HEAD_SHARD = 3 };
int enqueue_step(reng_model* m, int mode, int M, int slot, int head, cudaStream_t st, int* nk) {
    const int before = m->launches;
    TRY(k_embed_launch(m, mode, M, slot, st));
    for (int l = 0; l < m->L; l++) {
        TRY(k_qkv_launch(m, l, M, st));
        TRY(k_attn_launch(m, l, M, mode, st));
        TRY(k_proj_launch(m, l, M, 0, st));
        TRY(k_gateup_launch(m, l, M, st));
        TRY(k_proj_launch(m, l, M, 1, st));
    }
    if (head == HEAD_ALL) TRY(k_head_launch(m, mode, M, slot, st));
    else if (head == HEAD_SHARD) TRY(k_head_launch(m, mode, M, slot, st, 0, true));
    else if (head == HEAD_LAST) TRY(k_head_launch(m, mode, 1, slot, st, M - 1));
    if (nk) *nk = m->launches - before;
    return RENG_OK;
}

// One decode step (rows = the B slots) captured as a CUDA graph.
int capture_step(reng_model* m, int head, cudaGraphExec_t* out, int* nk) {
    cudaGraph_t g = nullptr;
    CU(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_step(m, 0, m->B, 0, head, m->st, nk);
    cudaError_t e = cudaStreamEndCapture(m->st, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return fail(RENG_E_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return fail(RENG_E_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
    return RENG_OK;
}

int build_graph(reng_model* m) {
    const bool shard = head_sharded(m);
    TRY(capture_step(m, shard ? HEAD_SHARD : HEAD_ALL, &m->graph, &m->kernels_per_step));
    if (shard) TRY(capture_step(m, HEAD_ALL, &m->graph_full, nullptr));
    return RENG_OK;
}

void free_model(reng_model* m) {
    if (!m) return;
    cudaSetDevice(m->dev);
    if (m->st) cudaStreamSynchronize(m->st);
    if (m->graph) cudaGraphExecDestroy(m->graph);
    if (m->graph_full) cudaGraphExecDestroy(m->graph_full);
    tp_destroy(m);
    for (void* p : m->allocs) cudaFree(p);
    if (m->pinned) cudaFreeHost(m->pinned);
    if (m->st) cudaStreamDestroy(m->st);
    delete m;
}

int create(const reng_model_desc* d, const reng_layer_weights* layers, const uint16_t* embed,
           const uint16_t* lm_head, const float* final_gamma, const float* rope_sin,
           const float* rope_cos, int mem, reng_model* m) {
    m->d = *d;
    m->d.nccl_id = nullptr;
    m->dev = d->device;
    CU(cudaSetDevice(m->dev));
    CU(cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking));
    m->sms = num_sms(m->dev);
    CU(gemv_prepare());
    CU(gemv8_prepare());
    CU(gemm_prepare());
    CU(attn_ring_prepare());
    m->rank = d->tp_rank;
    m->world = d->tp_world;
    m->w8 = d->weights == RENG_WEIGHTS_FP8_E4M3 ? 1 : 0;
    m->qk_norm = d->qk_norm == 1;
    // the attention scale rides on wq (and bq), or on the q norm gain
    // (scaled_wq, model.rs:148-157)
    const float wq_scale = m->qk_norm ? 1.0f : d->attn_scale;
    const int W = m->world, R = m->rank;
    m->hidden = d->hidden;
    m->L = d->n_layers;
    m->hd = d->head_dim;
    m->vocab = d->vocab;
    m->B = d->batch;
    m->cap = d->capacity;
    m->nh = d->n_heads / W;
    m->nkv = d->n_kv_heads / W;
    m->inter = d->inter / W;
    m->hpg = m->nh / m->nkv;
    m->q_dim = m->nh * m->hd;
    m->kv_dim = m->nkv * m->hd;
    const int q_full = d->n_heads * m->hd, kv_full = d->n_kv_heads * m->hd;
    const int H = m->hidden;
    if (W > 1) TRY(tp_init(m, d->nccl_id));

    // ---- tile maps ----
    const int ppt = m->hd / 16;  // pair tiles per head
    std::vector<int> qkv_map;
    for (int h = 0; h < m->nh; h++)
        for (int j = 0; j < ppt; j++) {
            for (int i = 0; i < 8; i++) qkv_map.push_back(h * m->hd + j * 8 + i);
            for (int i = 0; i < 8; i++) qkv_map.push_back(h * m->hd + j * 8 + i + m->hd / 2);
        }
    m->q_tiles = m->nh * ppt;
    for (int h = 0; h < m->nkv; h++)
        for (int j = 0; j < ppt; j++) {
            for (int i = 0; i < 8; i++) qkv_map.push_back(m->q_dim + h * m->hd + j * 8 + i);
            for (int i = 0; i < 8; i++) qkv_map.push_back(m->q_dim + h * m->hd + j * 8 + i + m->hd / 2);
        }
    m->k_tiles = m->nkv * ppt;
    for (int r = 0; r < m->kv_dim; r++) qkv_map.push_back(m->q_dim + m->kv_dim + r);
    std::vector<int> gu_map;
    for (int t = 0; t < m->inter / 8; t++) {
        for (int i = 0; i < 8; i++) gu_map.push_back(t * 8 + i);
        for (int i = 0; i < 8; i++) gu_map.push_back(m->inter + t * 8 + i);
    }

    // ---- staging buffer large enough for any one matrix ----
    size_t stage_el = std::max<size_t>((size_t)(m->q_dim + 2 * m->kv_dim) * H, (size_t)2 * m->inter * H);
    stage_el = std::max<size_t>(stage_el, (size_t)m->vocab * H);
    uint16_t* stage = nullptr;
    CU(cudaMalloc((void**)&stage, stage_el * 2));
    struct StageFree {
        uint16_t* p;
        ~StageFree() { cudaFree(p); }
    } sf{stage};

    m->layers.resize(m->L);
    std::vector<float> bias((size_t)m->q_dim + 2 * m->kv_dim);
    for (int l = 0; l < m->L; l++) {
        const reng_layer_weights& s = layers[l];
        RENG_CHECK_ARG(s.wq && s.wk && s.wv && s.wo && s.wg && s.wu && s.wd && s.g1 && s.g2,
                       "reng_model_create: layer " + std::to_string(l) + " has a NULL weight");
        if (d->has_qkv_bias)
            RENG_CHECK_ARG(s.bq && s.bk && s.bv, "reng_model_create: layer " + std::to_string(l) + " lacks a bias");
        LayerDev& w = m->layers[l];
        if (m->qk_norm)
            RENG_CHECK_ARG(s.qn && s.kn, "reng_model_create: layer " + std::to_string(l) + " lacks q/k norm gains");
        RENG_CHECK_ARG(s.no_rope == 0 || s.no_rope == 1, "reng_model_create: layer " + std::to_string(l) +
                                                             " no_rope must be 0 or 1");
        w.no_rope = s.no_rope == 1;
        m->any_no_rope = m->any_no_rope || w.no_rope;
        // q, k, v row blocks of this rank
        TRY(copy_matrix(stage, s.wq + (size_t)R * m->q_dim * H, m->q_dim, H, H, mem, m->st));
        TRY(copy_matrix(stage + (size_t)m->q_dim * H, s.wk + (size_t)R * m->kv_dim * H, m->kv_dim, H, H, mem, m->st));
        TRY(copy_matrix(stage + (size_t)(m->q_dim + m->kv_dim) * H, s.wv + (size_t)R * m->kv_dim * H, m->kv_dim, H, H,
                        mem, m->st));
        if (m->w8)
            TRY(pack_fp8(m, &w.wqkv, &w.sqkv, stage, m->q_dim + 2 * m->kv_dim, qkv_map, H, wq_scale, m->q_dim,
                         &m->qkv_tiles));
        else
            TRY(pack(m, &w.wqkv, stage, qkv_map, H, wq_scale, m->q_dim, &m->qkv_tiles));
        // o_proj column window
        TRY(copy_matrix(stage, s.wo + (size_t)R * m->q_dim, H, m->q_dim, q_full, mem, m->st));
        if (m->w8)
            TRY(pack_fp8(m, &w.wo, &w.so, stage, H, plain_map(H), m->q_dim, 1.f, 0, &m->o_tiles));
        else
            TRY(pack(m, &w.wo, stage, plain_map(H), m->q_dim, 0.f, 0, &m->o_tiles));
        // gate, up row blocks
        TRY(copy_matrix(stage, s.wg + (size_t)R * m->inter * H, m->inter, H, H, mem, m->st));
        TRY(copy_matrix(stage + (size_t)m->inter * H, s.wu + (size_t)R * m->inter * H, m->inter, H, H, mem, m->st));
        if (m->w8)
            TRY(pack_fp8(m, &w.wgu, &w.sgu, stage, 2 * m->inter, gu_map, H, 1.f, 0, &m->gu_tiles));
        else
            TRY(pack(m, &w.wgu, stage, gu_map, H, 0.f, 0, &m->gu_tiles));
        // down column window
        TRY(copy_matrix(stage, s.wd + (size_t)R * m->inter, H, m->inter, d->inter, mem, m->st));
        if (m->w8)
            TRY(pack_fp8(m, &w.wd, &w.sd, stage, H, plain_map(H), m->inter, 1.f, 0, &m->d_tiles));
        else
            TRY(pack(m, &w.wd, stage, plain_map(H), m->inter, 0.f, 0, &m->d_tiles));
        TRY(upload_f32(m, &w.g1, s.g1, H, mem));
        TRY(upload_f32(m, &w.g2, s.g2, H, mem));
        if (d->has_qkv_bias) {
            // q bias carries the attention scale (model.rs:2993-3002), in f32
            std::vector<float> hb((size_t)q_full + 2 * kv_full);
            auto fetch = [&](float* dst, const float* src, size_t n) -> int {
                if (mem == RENG_MEM_HOST) memcpy(dst, src, n * 4);
                else CU(cudaMemcpy(dst, src, n * 4, cudaMemcpyDeviceToHost));
                return RENG_OK;
            };
            TRY(fetch(hb.data(), s.bq, q_full));
            TRY(fetch(hb.data() + q_full, s.bk, kv_full));
            TRY(fetch(hb.data() + q_full + kv_full, s.bv, kv_full));
            for (int i = 0; i < m->q_dim; i++) bias[i] = hb[(size_t)R * m->q_dim + i] * wq_scale;
            for (int i = 0; i < m->kv_dim; i++) bias[m->q_dim + i] = hb[q_full + (size_t)R * m->kv_dim + i];
            for (int i = 0; i < m->kv_dim; i++)
                bias[m->q_dim + m->kv_dim + i] = hb[q_full + kv_full + (size_t)R * m->kv_dim + i];
            TRY(upload_f32(m, &w.bqkv, bias.data(), bias.size(), RENG_MEM_HOST));
            CU(cudaStreamSynchronize(m->st));
        }
        if (m->qk_norm) {
            // the attention scale rides on the q gain, in f32 (model.rs:2989-2991)
            std::vector<float> g((size_t)m->hd);
            if (mem == RENG_MEM_HOST) memcpy(g.data(), s.qn, g.size() * 4);
            else CU(cudaMemcpy(g.data(), s.qn, g.size() * 4, cudaMemcpyDeviceToHost));
            for (float& v : g) v *= d->attn_scale;
            TRY(upload_f32(m, &w.qn, g.data(), g.size(), RENG_MEM_HOST));
            TRY(upload_f32(m, &w.kn, s.kn, (size_t)m->hd, mem));
            CU(cudaStreamSynchronize(m->st));
        }
    }
    // LM head (replicated) and the embedding table
    RENG_CHECK_ARG(embed && lm_head && final_gamma && rope_sin && rope_cos, "reng_model_create: NULL table");
    TRY(copy_matrix(stage, lm_head, m->vocab, H, H, mem, m->st));
    TRY(pack(m, &m->lm, stage, plain_map(m->vocab), H, 0.f, 0, &m->lm_tiles));
    TRY(dalloc(m, &m->embed, (size_t)m->vocab * H));
    TRY(copy_matrix(m->embed, embed, m->vocab, H, H, mem, m->st));
    TRY(upload_f32(m, &m->final_gamma, final_gamma, H, mem));
    TRY(upload_f32(m, &m->rope_cos, rope_cos, (size_t)m->cap * m->hd, mem));
    TRY(upload_f32(m, &m->rope_sin, rope_sin, (size_t)m->cap * m->hd, mem));
    if (m->qk_norm || m->any_no_rope) {  // identity rotation for the q/k/v launch: cos 1, sin 0
        const size_t n = (size_t)m->cap * m->hd;
        TRY(upload_f32(m, &m->rope_sin_id, nullptr, n, RENG_MEM_HOST));
        TRY(dalloc(m, &m->rope_cos_id, n));
        k_fill_f32<<<m->sms * 4, 256, 0, m->st>>>(m->rope_cos_id, n, 1.0f);
        CU(cudaGetLastError());
    }

    // ---- KV cache and work buffers ----
    m->layer_kv = (size_t)m->B * m->nkv * m->cap * m->hd;
    TRY(dalloc(m, &m->kcache, m->layer_kv * m->L));
    TRY(dalloc(m, &m->vcache, m->layer_kv * m->L));
    CU(cudaMemsetAsync(m->kcache, 0, m->layer_kv * m->L * 2, m->st));
    CU(cudaMemsetAsync(m->vcache, 0, m->layer_kv * m->L * 2, m->st));
    const int MR = kBlockRows;
    TRY(dalloc(m, &m->x_res, (size_t)MR * H));
    TRY(dalloc(m, &m->qbuf, (size_t)MR * m->q_dim));
    TRY(dalloc(m, &m->xn, (size_t)MR * H));
    TRY(dalloc(m, &m->attn, (size_t)MR * m->q_dim));
    TRY(dalloc(m, &m->act, (size_t)MR * m->inter));
    TRY(dalloc(m, &m->logits, (size_t)MR * m->vocab));
    TRY(dalloc(m, &m->ss, (size_t)kSsStride * MR));
    TRY(dalloc(m, &m->part, (size_t)MR * H));
    TRY(dalloc(m, &m->row_slot, MR));
    TRY(dalloc(m, &m->row_pos, MR));
    TRY(dalloc(m, &m->pos, m->B));
    TRY(dalloc(m, &m->step, 1));
    TRY(dalloc(m, &m->err, 1));
    CU(cudaMemsetAsync(m->err, 0, 4, m->st));
    TRY(dalloc(m, &m->ids_ring, (size_t)(m->cap + 1) * m->B));
    TRY(dalloc(m, &m->prefill_ids, MR));
    TRY(dalloc(m, &m->next_id, 1));
    CU(cudaMemsetAsync(m->pos, 0, (size_t)m->B * 4, m->st));
    CU(cudaMemsetAsync(m->step, 0, 4, m->st));
    CU(cudaMemsetAsync(m->x_res, 0, (size_t)MR * H * 2, m->st));
    CU(cudaMemsetAsync(m->ss, 0, (size_t)kSsStride * MR * 4, m->st));

    // launch shapes
    const int kch = (H + kChunkK - 1) / kChunkK;
    const int kcs[5] = {proj_kc(m, H), proj_kc(m, m->q_dim), proj_kc(m, H), proj_kc(m, m->inter), kch};
    for (int k = 0; k < 5; k++) pick_shape(m, k, kcs[k], &m->shape[k][0], &m->shape[k][1]);
    {
        const char* v = getenv("RENG_GEMV8");  // a tuning knob: 0 keeps the shared-memory GEMV
        m->gemv8 = !(v && atoi(v) == 0);
    }
    m->lm_grid = m->sms * 32;  // an upper bound of the LM head's CTAs (GEMV grid, GEMM super-tiles)
    TRY(dalloc(m, &m->am_count, 1));
    CU(cudaMemsetAsync(m->am_count, 0, 4, m->st));
    // split-K partials: at most two CTAs per SM of 128 rows x N <= 64
    m->gpart_floats = (size_t)2 * m->sms * 128 * 64;
    TRY(dalloc(m, &m->gpart, m->gpart_floats));
    TRY(dalloc(m, &m->gcnt, (size_t)kGemmCntMax));
    CU(cudaMemsetAsync(m->gcnt, 0, (size_t)kGemmCntMax * 4, m->st));
    TRY(dalloc(m, &m->am_key, (size_t)kBlockRows));
    CU(cudaMemsetAsync(m->am_key, 0, (size_t)kBlockRows * 8, m->st));
    CU(cudaMallocHost((void**)&m->pinned, sizeof(uint32_t) * kPinnedWords));
    m->host_pos.assign(m->B, 0);
    CU(cudaStreamSynchronize(m->st));
    TRY(build_graph(m));
    return RENG_OK;
}

// Prompt rows per prefill block: kBlockRows (the GEMM path, FP8 weights
// included); RENG_PREFILL_ROWS lowers it (a tuning knob).
int prefill_rows(const reng_model* m) {
    int r = kBlockRows;
    const char* v = getenv("RENG_PREFILL_ROWS");
    if (v) {
        const int x = atoi(v);
        if (x >= 1 && x < r) r = x;
    }
    return r;
}

int check_model(const reng_model* m) {
    RENG_CHECK_ARG(m != nullptr, "model is NULL");
    return RENG_OK;
}

int sync_pos(reng_model* m) {
    int* hp = reinterpret_cast<int*>(m->pinned) + kPinnedPos;
    for (int b = 0; b < m->B; b++) hp[b] = m->host_pos[b];
    CU(cudaMemcpyAsync(m->pos, hp, (size_t)m->B * 4, cudaMemcpyHostToDevice, m->st));
    CU(cudaStreamSynchronize(m->st));
    return RENG_OK;
}

// The device error word of the bounded waits: RENG_E_TIMEOUT if a kernel
// gave up on a wait (its results are then invalid).  Synchronises.
int check_device_error(reng_model* m) {
    int* h = reinterpret_cast<int*>(m->pinned) + kPinnedErr;
    CU(cudaMemcpyAsync(h, m->err, 4, cudaMemcpyDeviceToHost, m->st));
    CU(cudaStreamSynchronize(m->st));
    if (*h != 0) {
        const int code = *h;
        CU(cudaMemsetAsync(m->err, 0, 4, m->st));
        // a launch that gave up may leave arrival counts and argmax keys mid-count
        CU(cudaMemsetAsync(m->gcnt, 0, (size_t)kGemmCntMax * 4, m->st));
        CU(cudaMemsetAsync(m->am_key, 0, (size_t)kBlockRows * 8, m->st));
        CU(cudaMemsetAsync(m->am_count, 0, 4, m->st));
        CU(cudaStreamSynchronize(m->st));
        return fail(code, code == RENG_E_INVAL
                              ? "a token id on the device was outside the vocabulary; the results are invalid"
                              : "a kernel of the step gave up on a bounded wait; the results are invalid");
    }
    return RENG_OK;
}

void bf16_to_f32_host(const uint16_t* s, float* d, size_t n) {
    for (size_t i = 0; i < n; i++) {
        uint32_t u = (uint32_t)s[i] << 16;
        memcpy(&d[i], &u, 4);
    }
}

}  // namespace

extern "C" int reng_model_create(const reng_model_desc* desc, const reng_layer_weights* layers,
                                 const uint16_t* embed, const uint16_t* lm_head,
                                 const float* final_gamma, const float* rope_sin,
                                 const float* rope_cos, int mem, reng_model** out) {
    RENG_CHECK_ARG(out != nullptr, "reng_model_create: out is NULL");
    *out = nullptr;
    TRY(validate(desc));
    RENG_CHECK_ARG(layers != nullptr, "reng_model_create: layers is NULL");
    RENG_CHECK_ARG(mem == RENG_MEM_HOST || mem == RENG_MEM_DEVICE, "reng_model_create: bad mem");
    if (desc->tp_world > 1) RENG_CHECK_ARG(desc->nccl_id != nullptr, "reng_model_create: tp_world > 1 needs nccl_id");
    reng_model* m = new (std::nothrow) reng_model();
    if (!m) return fail(RENG_E_NOMEM, "reng_model_create: host allocation");
    int rc = create(desc, layers, embed, lm_head, final_gamma, rope_sin, rope_cos, mem, m);
    if (rc) {
        std::string msg = reng_last_error();
        free_model(m);
        set_error(msg);
        return rc;
    }
    *out = m;
    return RENG_OK;
}

extern "C" int reng_model_destroy(reng_model* m) {
    if (m) free_model(m);
    return RENG_OK;
}

extern "C" int reng_model_prefill(reng_model* m, int slot, const uint32_t* ids, int n,
                                  uint32_t* next_id, float* last_logits, float* all_logits) {
    TRY(check_model(m));
    RENG_CHECK_ARG(slot >= 0 && slot < m->B, "reng_model_prefill: slot out of range");
    RENG_CHECK_ARG(ids != nullptr && n >= 1, "reng_model_prefill: empty prompt");
    RENG_CHECK_ARG((int64_t)m->host_pos[slot] + n <= m->cap,
                   "reng_model_prefill: " + std::to_string(m->host_pos[slot]) + " + " + std::to_string(n) +
                       " positions overflow the capacity " + std::to_string(m->cap));
    for (int i = 0; i < n; i++)
        RENG_CHECK_ARG(ids[i] < (uint32_t)m->vocab, "reng_model_prefill: token id " + std::to_string(ids[i]) +
                                                        " out of range");
    CU(cudaSetDevice(m->dev));
    std::vector<uint16_t> hl;
    const int block = prefill_rows(m);
    for (int b0 = 0; b0 < n; b0 += block) {
        const int M = std::min(block, n - b0);
        const bool last = b0 + M == n;
        memcpy(m->pinned, ids + b0, (size_t)M * 4);
        CU(cudaMemcpyAsync(m->prefill_ids, m->pinned, (size_t)M * 4, cudaMemcpyHostToDevice, m->st));
        // positions of this block: pos[slot] on the device is the block base
        const int head = all_logits ? HEAD_ALL : (last ? HEAD_LAST : HEAD_NONE);
        TRY(enqueue_step(m, 1, M, slot, head, m->st, nullptr));
        m->host_pos[slot] += M;
        TRY(sync_pos(m));  // also orders the pinned buffer reuse
        if (all_logits) {
            hl.resize((size_t)M * m->vocab);
            CU(cudaMemcpy(hl.data(), m->logits, hl.size() * 2, cudaMemcpyDeviceToHost));
            bf16_to_f32_host(hl.data(), all_logits + (size_t)b0 * m->vocab, hl.size());
        }
        if (last) {
            if (last_logits) {
                hl.resize((size_t)m->vocab);
                const size_t row = head == HEAD_ALL ? (size_t)(M - 1) : 0;
                CU(cudaMemcpy(hl.data(), m->logits + row * m->vocab, (size_t)m->vocab * 2,
                              cudaMemcpyDeviceToHost));
                bf16_to_f32_host(hl.data(), last_logits, m->vocab);
            }
            uint32_t id = 0;
            CU(cudaMemcpy(&id, m->next_id, 4, cudaMemcpyDeviceToHost));
            if (next_id) *next_id = id;
        }
    }
    return check_device_error(m);
}

static int decode_common(reng_model* m, int n, cudaStream_t st) {
    for (int i = 0; i < n; i++) CU(cudaGraphLaunch(m->graph, st));
    return RENG_OK;
}

extern "C" int reng_model_decode_device(reng_model* m, const uint32_t* seeds, int n, uint32_t* ids_out,
                                        void* stream) {
    TRY(check_model(m));
    RENG_CHECK_ARG(seeds && ids_out && n >= 1, "reng_model_decode_device: bad arguments");
    for (int b = 0; b < m->B; b++)
        RENG_CHECK_ARG((int64_t)m->host_pos[b] + n <= m->cap,
                       "reng_model_decode_device: slot " + std::to_string(b) + " would overflow the capacity");
    CU(cudaSetDevice(m->dev));
    cudaStream_t st = (cudaStream_t)stream;
    CU(cudaMemcpyAsync(m->ids_ring, seeds, (size_t)m->B * 4, cudaMemcpyDeviceToDevice, st));
    CU(cudaMemsetAsync(m->step, 0, 4, st));
    TRY(decode_common(m, n, st));
    CU(cudaMemcpyAsync(ids_out, m->ids_ring + m->B, (size_t)n * m->B * 4, cudaMemcpyDeviceToDevice, st));
    for (int b = 0; b < m->B; b++) m->host_pos[b] += n;
    return RENG_OK;
}

extern "C" int reng_model_decode(reng_model* m, const uint32_t* seeds, int n, uint32_t* ids_out) {
    TRY(check_model(m));
    RENG_CHECK_ARG(seeds && ids_out && n >= 1, "reng_model_decode: bad arguments");
    for (int b = 0; b < m->B; b++) {
        RENG_CHECK_ARG((int64_t)m->host_pos[b] + n <= m->cap,
                       "reng_model_decode: slot " + std::to_string(b) + " at " + std::to_string(m->host_pos[b]) +
                           " + " + std::to_string(n) + " overflows the capacity " + std::to_string(m->cap));
        RENG_CHECK_ARG(seeds[b] < (uint32_t)m->vocab, "reng_model_decode: seed id out of range");
    }
    CU(cudaSetDevice(m->dev));
    EventSet evs;
    CU(evs.create(4));
    cudaEvent_t* ev = evs.e;
    CU(cudaEventRecord(ev[0], m->st));
    memcpy(m->pinned, seeds, (size_t)m->B * 4);
    CU(cudaMemcpyAsync(m->ids_ring, m->pinned, (size_t)m->B * 4, cudaMemcpyHostToDevice, m->st));
    CU(cudaMemsetAsync(m->step, 0, 4, m->st));
    CU(cudaEventRecord(ev[1], m->st));
    TRY(decode_common(m, n, m->st));
    CU(cudaEventRecord(ev[2], m->st));
    CU(cudaMemcpyAsync(ids_out, m->ids_ring + m->B, (size_t)n * m->B * 4, cudaMemcpyDeviceToHost, m->st));
    CU(cudaEventRecord(ev[3], m->st));
    CU(cudaEventSynchronize(ev[3]));
    cudaEventElapsedTime(&m->times.upload_ms, ev[0], ev[1]);
    cudaEventElapsedTime(&m->times.device_ms, ev[1], ev[2]);
    cudaEventElapsedTime(&m->times.readback_ms, ev[2], ev[3]);
    m->times.steps = n;
    m->times.kernels_per_step = m->kernels_per_step;
    for (int b = 0; b < m->B; b++) m->host_pos[b] += n;
    return check_device_error(m);
}

extern "C" int reng_model_step_logits(reng_model* m, const uint32_t* ids, float* logits, uint32_t* next_ids) {
    TRY(check_model(m));
    RENG_CHECK_ARG(ids != nullptr, "reng_model_step_logits: ids is NULL");
    for (int b = 0; b < m->B; b++) {
        RENG_CHECK_ARG((int64_t)m->host_pos[b] + 1 <= m->cap, "reng_model_step_logits: capacity overflow");
        RENG_CHECK_ARG(ids[b] < (uint32_t)m->vocab, "reng_model_step_logits: id out of range");
    }
    CU(cudaSetDevice(m->dev));
    memcpy(m->pinned, ids, (size_t)m->B * 4);
    CU(cudaMemcpyAsync(m->ids_ring, m->pinned, (size_t)m->B * 4, cudaMemcpyHostToDevice, m->st));
    CU(cudaMemsetAsync(m->step, 0, 4, m->st));
    CU(cudaGraphLaunch(m->graph_full ? m->graph_full : m->graph, m->st));
    std::vector<uint16_t> hl((size_t)m->B * m->vocab);
    CU(cudaMemcpyAsync(hl.data(), m->logits, hl.size() * 2, cudaMemcpyDeviceToHost, m->st));
    CU(cudaMemcpyAsync(m->pinned, m->ids_ring + m->B, (size_t)m->B * 4, cudaMemcpyDeviceToHost, m->st));
    CU(cudaStreamSynchronize(m->st));
    if (logits) bf16_to_f32_host(hl.data(), logits, hl.size());
    if (next_ids) memcpy(next_ids, m->pinned, (size_t)m->B * 4);
    for (int b = 0; b < m->B; b++) m->host_pos[b] += 1;
    return check_device_error(m);
}

extern "C" int reng_model_reset(reng_model* m, int slot) {
    TRY(check_model(m));
    RENG_CHECK_ARG(slot >= -1 && slot < m->B, "reng_model_reset: slot out of range");
    CU(cudaSetDevice(m->dev));
    CU(cudaStreamSynchronize(m->st));
    for (int b = 0; b < m->B; b++)
        if (slot < 0 || slot == b) m->host_pos[b] = 0;
    return sync_pos(m);
}

extern "C" int reng_model_position(const reng_model* m, int slot, int* pos) {
    TRY(check_model(m));
    RENG_CHECK_ARG(pos && slot >= 0 && slot < m->B, "reng_model_position: bad slot");
    *pos = m->host_pos[slot];
    return RENG_OK;
}

extern "C" int reng_model_tp_exchange(reng_model* m, int* kind) {
    TRY(check_model(m));
    RENG_CHECK_ARG(kind != nullptr, "reng_model_tp_exchange: NULL");
    *kind = tp_exchange_kind(m);
    return RENG_OK;
}

extern "C" int reng_model_device_bytes(const reng_model* m, uint64_t* bytes) {
    TRY(check_model(m));
    RENG_CHECK_ARG(bytes != nullptr, "reng_model_device_bytes: NULL");
    *bytes = m->bytes;
    return RENG_OK;
}

extern "C" int reng_model_last_times(const reng_model* m, reng_step_times* t) {
    TRY(check_model(m));
    RENG_CHECK_ARG(t != nullptr, "reng_model_last_times: NULL");
    *t = m->times;
    return RENG_OK;
}

extern "C" int reng_model_time_kernels_rows(reng_model* m, int rows, int iters, float* ms_out) {
    TRY(check_model(m));
    RENG_CHECK_ARG(ms_out != nullptr && iters >= 1, "reng_model_time_kernels: bad arguments");
    RENG_CHECK_ARG(rows >= 0 && rows <= prefill_rows(m), "reng_model_time_kernels_rows: rows must be in [0, " +
                                                            std::to_string(prefill_rows(m)) + "]");
    RENG_CHECK_ARG((int64_t)m->host_pos[0] + rows <= m->cap,
                   "reng_model_time_kernels_rows: slot 0 has no room for the block");
    CU(cudaSetDevice(m->dev));
    CU(cudaStreamSynchronize(m->st));
    const int mode = rows > 0 ? 1 : 0;
    const int M = rows > 0 ? rows : m->B;
    EventSet evs;
    CU(evs.create(2));
    cudaEvent_t e0 = evs.e[0], e1 = evs.e[1];
    // rows as the decode step sees them, or a prefill block of slot 0 at
    // its current position
    if (rows > 0) TRY(sync_pos(m));
    TRY(k_embed_launch(m, mode, M, 0, m->st));
    for (int kind = 0; kind < RENG_KERNEL_KINDS; kind++) {
        // one untimed pass, then `iters` launches cycling over the layers
        for (int pass = 0; pass < 2; pass++) {
            const int n = pass == 0 ? std::min(iters, m->L) : iters;
            if (pass == 1) CU(cudaEventRecord(e0, m->st));
            for (int i = 0; i < n; i++) {
                const int l = i % m->L;
                switch (kind) {
                    case 0: TRY(k_qkv_launch(m, l, M, m->st)); break;
                    case 1: TRY(k_attn_launch(m, l, M, mode, m->st)); break;
                    case 2: TRY(k_proj_launch(m, l, M, 0, m->st)); break;
                    case 3: TRY(k_gateup_launch(m, l, M, m->st)); break;
                    case 4: TRY(k_proj_launch(m, l, M, 1, m->st)); break;
                    default: TRY(k_head_launch(m, 1, M, 0, m->st)); break;
                }
            }
            if (pass == 1) CU(cudaEventRecord(e1, m->st));
        }
        CU(cudaEventSynchronize(e1));
        float ms = 0.f;
        CU(cudaEventElapsedTime(&ms, e0, e1));
        ms_out[kind] = ms / (float)iters;
    }
    TRY(check_device_error(m));
    // the QKV launches rewrote the cache row at each slot's last position
    // (or the block's rows) with other activations: the cached prefix is no
    // longer valid
    for (int b = 0; b < m->B; b++) m->host_pos[b] = 0;
    return sync_pos(m);
}

extern "C" int reng_model_time_kernels(reng_model* m, int iters, float* ms_out) {
    return reng_model_time_kernels_rows(m, 0, iters, ms_out);
}

extern "C" int reng_model_time_exchange(reng_model* m, int iters, float* ms_out) {
    TRY(check_model(m));
    RENG_CHECK_ARG(ms_out != nullptr && iters >= 1, "reng_model_time_exchange: bad arguments");
    if (m->world < 2) return fail(RENG_E_STATE, "reng_model_time_exchange: the model is not tensor-parallel");
    CU(cudaSetDevice(m->dev));
    CU(cudaStreamSynchronize(m->st));
    const int M = m->B;
    // the exchange of M rows exactly as a decode step issues it after
    // o_proj / down_proj (the peer all-reduce for M <= kMaxRows, otherwise
    // NCCL + the residual kernel), on whatever partials the buffer holds;
    // `iters` of them captured in one graph as the step graph holds them,
    // so the time is the device's, not the host's launch rate
    auto one = [&]() -> int {
        if (tp_p2p(m, M)) {
            CU(launch_tp_ar_residual(m, m->part, M, m->st));
        } else {
            CU(tp_allreduce(m, m->part, (size_t)M * m->hidden, m->st));
            CU(launch_tp_residual(m, m->part, M, false, m->st));
        }
        return RENG_OK;
    };
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    CU(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
    int rc = RENG_OK;
    for (int i = 0; i < iters && rc == RENG_OK; i++) rc = one();
    cudaError_t e = cudaStreamEndCapture(m->st, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return fail(RENG_E_CUDA, std::string("exchange capture: ") + cudaGetErrorString(e));
    e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return fail(RENG_E_CUDA, std::string("exchange instantiate: ") + cudaGetErrorString(e));
    struct Exec {
        cudaGraphExec_t x;
        ~Exec() { cudaGraphExecDestroy(x); }
    } hold{ge};
    EventSet evs;
    CU(evs.create(2));
    CU(cudaGraphLaunch(ge, m->st));  // untimed: every rank's first replay meets the others
    CU(cudaEventRecord(evs.e[0], m->st));
    CU(cudaGraphLaunch(ge, m->st));
    CU(cudaEventRecord(evs.e[1], m->st));
    CU(cudaEventSynchronize(evs.e[1]));
    float ms = 0.f;
    CU(cudaEventElapsedTime(&ms, evs.e[0], evs.e[1]));
    *ms_out = ms / (float)iters;
    TRY(check_device_error(m));
    // the residual stream took the stale partials: the cached prefix is no
    // longer the one the slots' positions describe
    for (int b = 0; b < m->B; b++) m->host_pos[b] = 0;
    return sync_pos(m);
}


// ------------------------------------------------------------------- TP --
// Tensor parallelism is wired through NCCL in tp.cu; these accessors let it
// reach the model's buffers without exposing the struct.
namespace reng {
void* tp_handle(reng_model* m) { return m->nccl; }
void tp_set_handle(reng_model* m, void* h) { m->nccl = h; }
int tp_rank_of(reng_model* m) { return m->rank; }
int tp_world_of(reng_model* m) { return m->world; }
int tp_device_of(reng_model* m) { return m->dev; }
uint16_t* tp_x_res(reng_model* m) { return m->x_res; }
float* tp_ss(reng_model* m) { return m->ss; }
int tp_hidden(reng_model* m) { return m->hidden; }
int* tp_err(reng_model* m) { return m->err; }
}  // namespace reng
