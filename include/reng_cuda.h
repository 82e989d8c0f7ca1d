/*
 * reng_cuda.h -- the C ABI of libreng_cuda.so, the B200 (sm_100a) decoder
 * inference path that stands in for the reference engine's `reng-synapse`
 * crate and `reng-fp8`'s quantize API.
 *
 * The reference has no plugin API: its seam is the Rust API of
 * `reng-synapse` as `reng-model` consumes it.  Each entry point below names
 * the reference interface it replaces (paths relative to the reference
 * project).  A Rust `reng-cuda` crate binds these symbols one-to-one; the
 * ctypes binding used by this repository's tests and bench is
 * reciprocating-engine_b200/reng/_lib.py.
 *
 * Conventions
 *  - Every function returns RENG_OK (0) or a negative RENG_E_* code; the
 *    message of the last failure on the calling thread is returned by
 *    reng_last_error().  Nothing aborts: shape misuse that the reference
 *    answers with a panic (assert!) is RENG_E_INVAL here.
 *  - Weights are bf16 bit patterns (uint16_t) in the checkpoint's own
 *    [out, in] row-major layout; gains and biases are f32.
 *  - `mem` says where caller buffers live: RENG_MEM_HOST (pageable or
 *    pinned host memory; copies happen inside the call) or RENG_MEM_DEVICE
 *    (device pointers on the current device, used in place).
 *  - `stream` is a cudaStream_t (NULL = the legacy default stream).
 */
#ifndef RENG_CUDA_H
#define RENG_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RENG_OK 0
#define RENG_E_INVAL (-1)       /* bad argument or shape */
#define RENG_E_CUDA (-2)        /* a CUDA runtime call failed */
#define RENG_E_NOMEM (-3)       /* a device or host allocation failed */
#define RENG_E_STATE (-4)       /* call not valid in the object's state */
#define RENG_E_UNSUPPORTED (-5) /* configuration this build does not run */
#define RENG_E_NCCL (-6)        /* an NCCL call failed */
#define RENG_E_TIMEOUT (-7)     /* a bounded device wait ran out */

#define RENG_MEM_DEVICE 0
#define RENG_MEM_HOST 1

/* Message of the last failure on this thread ("" if none). */
const char *reng_last_error(void);

/* ABI version: (major << 16) | minor.  Minor 2 added reng_model_desc.qk_norm
 * and reng_layer_weights.qn / kn / no_rope (callers built against minor 1
 * pass structs that are too short); minor 3 added
 * reng_model_time_kernels_rows and removed reng_model_trace_step. */
int reng_version(void);

/* Number of CUDA devices (replaces reng-hal's Gaudi accel discovery,
 * crates/reng-hal/src/lib.rs:62).  A host without a CUDA driver or device
 * has 0 devices, not an error, as the reference's enumeration is empty on a
 * host without the accel class. */
int reng_device_count(int *count);

/* One device's record (the role of reng-hal's GaudiDevice: index, kind,
 * PCI address, silicon revision; crates/reng-hal/src/lib.rs:24-33). */
typedef struct reng_device_info {
    int32_t ordinal;        /* CUDA device ordinal */
    char name[96];          /* the device's product name */
    char pci_bus_id[32];    /* "0000:cc:00.0" form */
    uint64_t total_bytes;   /* device memory */
    int32_t sm_count;       /* streaming multiprocessors */
    int32_t cc_major, cc_minor; /* compute capability (10.0 on B200) */
} reng_device_info;
int reng_device_info_get(int device, reng_device_info *out);

/* ===================================================== FP8 quantizer ===
 * Replaces reng_fp8::quantize_with (crates/reng-fp8/src/lib.rs:519-563)
 * and the Fp8Format / Scaling enums (lib.rs:53-147, 240-275).
 */
#define RENG_FP8_E4M3 0 /* 1-4-3, bias 7, max finite 240 (0x77), Gaudi range */
#define RENG_FP8_E5M2 1 /* 1-5-2, bias 15, max finite 57344 (0x7b) */

#define RENG_SCALING_PCS 0  /* per-output-channel absmax scale */
#define RENG_SCALING_HW 1   /* one power-of-16 factor as an exponent bias */
#define RENG_SCALING_UNIT 2 /* no scaling */

/*
 * Quantize a bf16 [rows, cols] matrix: per-row absmax, scale
 * absmax / (max_finite * backoff) (1.0 for an all-zero row), codes
 * encode(f32(w) / scale) with round-to-nearest-even and saturation to the
 * format's largest finite value, NaN -> sign|0x7f.  Bit-exact with
 * reng_fp8::quantize_with.  `codes` is [rows, cols] u8, `scales` is [rows]
 * f32, `*exp_bias` receives the exponent bias (a host pointer in both
 * memory modes).  rows, cols > 0 and a positive finite backoff are
 * required (the reference panics otherwise; RENG_E_INVAL here).
 */
int reng_fp8_quantize(const uint16_t *w, int64_t rows, int64_t cols, int fmt, int scaling,
                      float backoff, uint8_t *codes, float *scales, uint32_t *exp_bias,
                      int mem, void *stream);

/*
 * reng_fp8_quantize for callers that must not allocate device memory: the
 * same results, host buffers in and out (w, codes, scales, exp_bias as in
 * reng_fp8_quantize with RENG_MEM_HOST), but the device staging lives in
 * one fixed array inside the library instead of memory allocated per call.
 * Meant for code that runs while another allocator has reserved the GPU's
 * memory, or that must not enter the CUDA allocator on its path (no
 * cudaMalloc, cudaFree or allocating library call is made here).
 * Limits: rows <= 65,536 and rows * cols <= 2,097,152; larger matrices are
 * refused with RENG_E_INVAL.  Every GPU that loads the library holds the
 * 6.25 MiB array until exit.  The first call on a device looks up the
 * array's device address and keeps it for the process; make that first call
 * before any stream capture.  The kept address belongs to the device's
 * primary context: after cudaDeviceReset on that device, or when calling
 * from another context on it, the array may have moved and this entry must
 * not be used.
 * All calls on a device share the array: calls that overlap on the GPU (two
 * streams, two host threads) race and must be serialised by the caller.
 * The call returns after its copies back to the host are complete.
 * No counterpart in the reference (its quantizer is host code).
 */
int reng_fp8_quantize_noalloc(const uint16_t *w, int64_t rows, int64_t cols, int fmt, int scaling,
                              float backoff, uint8_t *codes, float *scales, uint32_t *exp_bias,
                              void *stream);

/* Encode n f32 values to fp8 codes, reng_fp8::encode
 * (crates/reng-fp8/src/lib.rs:154-201).  Device pointers. */
int reng_fp8_encode(const float *x, int64_t n, int fmt, uint8_t *codes, void *stream);

/* Decode n codes to f32, reng_fp8::decode (lib.rs:205-225). Device pointers. */
int reng_fp8_decode(const uint8_t *codes, int64_t n, int fmt, float *out, void *stream);

/* ========================================================== decoder ===
 * Replaces reng_synapse::CachedModel (crates/reng-synapse/src/cached.rs:
 * 128-1073), BatchedModel (batched.rs:95-1241) and tp::TpModel
 * (tp.rs:226-804), fed by the weight views of reng_synapse::ModelWeights /
 * LayerWeights (model.rs:2688-2733, layer.rs:16-136).
 */
typedef struct reng_model reng_model;

#define RENG_WEIGHTS_BF16 0     /* bf16 projections */
#define RENG_WEIGHTS_FP8_E4M3 1 /* projections quantized on the device at
                                   create time: E4M3, per-channel scales,
                                   backoff 1.0 (reng_fp8_quantize) */

typedef struct reng_model_desc {
    int32_t hidden;         /* hidden_size */
    int32_t inter;          /* intermediate_size */
    int32_t n_layers;       /* num_hidden_layers */
    int32_t n_heads;        /* num_attention_heads */
    int32_t n_kv_heads;     /* num_key_value_heads */
    int32_t head_dim;       /* head_dim */
    int32_t vocab;          /* vocab_size */
    float eps;              /* rms_norm_eps */
    float attn_scale;       /* softmax scale, folded into bf16 wq (model.rs:151-157) */
    int32_t has_qkv_bias;   /* q/k/v biases present (Qwen2) */
    int32_t weights;        /* RENG_WEIGHTS_* */
    int32_t batch;          /* decode slots B (1 = CachedModel, >1 = BatchedModel) */
    int32_t capacity;       /* KV positions per slot */
    int32_t tp_rank;        /* tensor-parallel rank (0 without TP) */
    int32_t tp_world;       /* tensor-parallel world size (1 without TP) */
    int32_t device;         /* CUDA device ordinal the model lives on */
    const uint8_t *nccl_id; /* 128-byte ncclUniqueId when tp_world > 1, else NULL */
    int32_t qk_norm;        /* 1: per-head RMSNorm of q and k before RoPE (Qwen3,
                               model.rs:2962-3010); the layers carry qn / kn
                               [head_dim] gains, and attn_scale rides on qn, not
                               on wq.  0 otherwise. */
} reng_model_desc;

/* One decoder layer's weights (layer.rs:16-136): bf16 [out, in] projections
 * and f32 vectors.  bq/bk/bv may be NULL when has_qkv_bias is 0.  With
 * tp_world > 1 these are the FULL (unsharded) matrices; the library copies
 * rank tp_rank's row blocks of q/k/v/gate/up and column windows of o/down
 * (reng-model/src/lib.rs:1155-1243). */
typedef struct reng_layer_weights {
    const uint16_t *wq, *wk, *wv, *wo; /* [q_dim,h] [kv_dim,h] [kv_dim,h] [h,q_dim] */
    const uint16_t *wg, *wu, *wd;      /* [inter,h] [inter,h] [h,inter] */
    const float *g1, *g2;              /* input_layernorm, post_attention_layernorm [h] */
    const float *bq, *bk, *bv;         /* [q_dim] [kv_dim] [kv_dim] or NULL */
    const float *qn, *kn;              /* [head_dim] q / k norm gains with qk_norm, else NULL */
    int32_t no_rope;                   /* 1: the layer rotates nothing (SmolLM3's NoPE layers,
                                          reng-model use_rope), else 0 */
} reng_layer_weights;

/*
 * Build a model: upload (or, for RENG_MEM_DEVICE, copy from device
 * buffers) and pack the weights, allocate the HBM-resident KV cache of
 * `batch` slots x `capacity` positions, and capture the decode step as a
 * CUDA graph.  rope_sin/rope_cos are the [capacity, head_dim] f32 tables
 * of reng-model's rope_caches (reng-model/src/lib.rs:2188-2216).  embed is
 * [vocab, hidden] bf16; lm_head may equal embed (tied).  Replaces
 * CachedModel::new (cached.rs:194), BatchedModel::new (batched.rs:161) and
 * TpModel::new (tp.rs:306).
 */
int reng_model_create(const reng_model_desc *desc, const reng_layer_weights *layers,
                      const uint16_t *embed, const uint16_t *lm_head,
                      const float *final_gamma, const float *rope_sin, const float *rope_cos,
                      int mem, reng_model **out);

int reng_model_destroy(reng_model *m);

/*
 * Append `n` prompt ids to slot `slot` and return the greedy next id (argmax
 * of the bf16 logits of the last position, first index of the max).  If
 * last_logits is not NULL it receives that position's `vocab` logits as f32
 * (the bf16 device values, widened).  `all_logits`, if not NULL, receives
 * [n, vocab] f32 logits of every position.  Host pointers.  Replaces
 * CachedModel::step_last_id / step_last / step (cached.rs:917-1072) and
 * BatchedModel::prefill_id / prefill (batched.rs:904-1021).
 */
int reng_model_prefill(reng_model *m, int slot, const uint32_t *ids, int n, uint32_t *next_id,
                       float *last_logits, float *all_logits);

/*
 * Greedy decode: every slot b appends seeds[b], then the device runs `n`
 * steps, each feeding the previous argmax back on the device, with no host
 * round trip between steps.  ids_out is [n, batch] (step-major).  Host
 * pointers; one copy in, one copy out.  Replaces CachedModel::step_ids /
 * loop_steps (cached.rs:752-835) and BatchedModel::run_ids / loop_steps
 * (batched.rs:1023-1151).
 */
int reng_model_decode(reng_model *m, const uint32_t *seeds, int n, uint32_t *ids_out);

/* The same with device-resident seeds [batch] and ids_out [n, batch], on
 * `stream`; asynchronous (no host synchronisation).  A seed outside the
 * vocabulary cannot be checked on the host: the gather reads row 0 for it and
 * the next synchronous call on the model returns RENG_E_INVAL. */
int reng_model_decode_device(reng_model *m, const uint32_t *seeds, int n, uint32_t *ids_out,
                             void *stream);

/*
 * One decode step that also returns the logits: every slot b appends ids[b];
 * logits [batch, vocab] f32 (bf16 device values) and next_ids [batch] are
 * written if not NULL.  Host pointers.  Replaces CachedModel::step_id_logits
 * (cached.rs) and BatchedModel::run_ids_logits / step (batched.rs).
 */
int reng_model_step_logits(reng_model *m, const uint32_t *ids, float *logits,
                           uint32_t *next_ids);

/* Forget slot `slot`'s cached prefix (-1: every slot).  CachedModel::reset
 * (cached.rs:840), BatchedModel::reset. */
int reng_model_reset(reng_model *m, int slot);

/* Positions held by slot `slot`.  CachedModel::position / BatchedModel::position. */
int reng_model_position(const reng_model *m, int slot, int *pos);

/* Device bytes held by the model (weights, KV cache, work buffers). */
int reng_model_device_bytes(const reng_model *m, uint64_t *bytes);

/* Wall-clock of the last reng_model_decode call split into its phases (ms):
 * upload, device steps, readback.  Mirrors RENG_STEP_TRACE (cached.rs:776-832). */
typedef struct reng_step_times {
    float upload_ms, device_ms, readback_ms;
    int32_t steps, kernels_per_step;
} reng_step_times;
int reng_model_last_times(const reng_model *m, reng_step_times *t);

/*
 * Diagnostic: mean device time (ms) of each kernel kind of the decode step,
 * launched alone on the model's stream `iters` times (CUDA events), cycling
 * over the layers so that no launch reads weights a previous one left in
 * L2.  ms_out[RENG_KERNEL_KINDS]: 0 qkv (rms1 + q/k/v + RoPE + KV write),
 * 1 attention, 2 o_proj (+ residual), 3 gate/up (rms2 + SwiGLU),
 * 4 down_proj (+ residual), 5 LM head (final rms + logits + argmax).
 * Rows are the B decode slots at their current positions.  It rewrites
 * cache rows, so every slot is reset (position 0) afterwards.  No reference
 * counterpart: the reference profiles through SynapseAI traces
 * (tools/profile/README.md).
 */
#define RENG_KERNEL_KINDS 6
int reng_model_time_kernels(reng_model *m, int iters, float *ms_out);
/* The same kinds at a prefill block of `rows` rows of slot 0 (rows > 0;
 * 0 is reng_model_time_kernels): the block starts at slot 0's position,
 * attention runs the prefill form and the LM head every row.  rows is at
 * most the engine's prefill block.  Every slot is reset afterwards. */
int reng_model_time_kernels_rows(reng_model *m, int rows, int iters, float *ms_out);

/* ==================================================== packed GEMM ===
 * y[m][r] = sum_k x[m][k] * w[r][k] (f32 out) through the tcgen05 GEMM the
 * model runs for steps of more than 8 rows: w (bf16 [rows][K], row-major)
 * is packed into the engine's swizzled 16 x 64 blocks, x (bf16 [M][K]) is
 * read by the tensor-memory-accelerator copy, the accumulator lives in
 * tensor memory.  Host buffers (mem RENG_MEM_HOST) or device buffers
 * (RENG_MEM_DEVICE).  1 <= M <= 1024 (N-tiles of 256 rows beyond 256),
 * K % 8 == 0.  splits = K splits (0:
 * the model's choice; > 0: that many CTAs of one cluster adding their
 * partials over shared memory; < 0: -splits plain CTAs adding theirs
 * through global scratch, the last to arrive in split order).  iters > 0:
 * the kernel alone is also launched iters more times and *ms_out gets its
 * mean duration (CUDA events).  The
 * reference's projections are SynapseAI graph matmuls (reng-synapse
 * src/model.rs:2960-3040); this entry exists so the kernel can be checked
 * and timed on its own.
 */
int reng_gemm_bf16(const uint16_t *w, int rows, int K, const uint16_t *x, int M, float *y, int splits,
                   int iters, float *ms_out, int mem);

/* ============================================== tensor parallelism ===
 * Replaces hccl::Rank::join's unique-id exchange (hccl.rs:580-637): rank 0
 * creates the id, the caller ships it to the other ranks (a file, a store),
 * each rank passes it in reng_model_desc.nccl_id.  The all-reduces after
 * o_proj and down_proj (tp.rs:709-793, hccl.rs:646) run inside the step.
 */
int reng_tp_unique_id(uint8_t out[128]);

/* How a tensor-parallel model exchanges its partials: 0 none (world 1),
 * 1 ncclAllReduce + a residual kernel, 2 the one-shot peer all-reduce over
 * NVLink fused with the residual (decode steps of up to 8 rows; prefill
 * blocks still use NCCL).  RENG_TP_P2P=0 in every rank's environment keeps
 * NCCL.  The reference exchanges through hcclAllReduce (hccl.rs:646-651). */
int reng_model_tp_exchange(reng_model *m, int *kind);

/* Diagnostic: mean device time (ms) of one partial exchange of the decode
 * step (the kind reng_model_tp_exchange names, for the model's B rows):
 * `iters` exchanges captured back to back in one CUDA graph, as the step
 * graph holds them, replayed once untimed and once under CUDA events.  Every
 * rank of the model must call it at the same time with the same iters (the
 * exchange waits on its peers).  It adds the partial buffer into the
 * residual stream, so every slot is reset (position 0) afterwards.
 * RENG_E_STATE for a model of world 1.  The reference measures its
 * all-reduce floor the same way, in isolation (hccl.rs:1330, 1363;
 * reng-ceiling strategy.rs:114-150). */
int reng_model_time_exchange(reng_model *m, int iters, float *ms_out);

/* Check of the exchange's failure path on one GPU: the peer all-reduce
 * kernel as rank 0 of two whose rank 1 never answers.  Its waits give up
 * after their bound (2 s) and it reports RENG_E_TIMEOUT, which this call
 * returns; the context stays usable (no fault, no hang).  Any other return
 * is a failure of the check.  The reference's counterpart is the HCCL
 * watchdog of hccl.rs:580-637. */
int reng_tp_peer_wait_check(int device);

#ifdef __cplusplus
}
#endif

#endif /* RENG_CUDA_H */
