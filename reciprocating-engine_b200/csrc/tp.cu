// Tensor parallelism: the NCCL communicator of a model and the all-reduce of
// the f32 o_proj / down_proj partials after each half-layer (the reference's
// TpModel, crates/reng-synapse/src/tp.rs:1-42 and :709-793, with its HCCL
// all-reduce, hccl.rs:477-506 / :646-651).
//
// Two exchanges:
//  * decode steps (rows <= kMaxRows): a one-shot all-reduce over NVLink
//    peer memory fused with the residual add.  Every rank owns a receive
//    area mapped into every other rank's address space (CUDA IPC handles,
//    exchanged once through the NCCL communicator).  CTA c of the kernel
//    takes hidden slice c: it stores its f32 partial slice into every peer's
//    area (plain peer stores over NVLink; no multicast), each value in one
//    8-byte word with the exchange's epoch, waits (bounded) until its own
//    elements' words from every peer carry that epoch, sums the W partials
//    in rank order (the same order on every rank, so every rank gets the
//    same bits), casts to bf16, adds the residual in bf16 and writes the
//    slice's norm partials.  One launch instead of an NCCL all-reduce and a
//    residual kernel.  Measured on B200 (Llama-8B TP2): a separate flag per
//    slice raised after a system-scope fence ended each exchange 10 us after
//    its start, the fence alone 3 us of it.
//  * prefill blocks (and worlds where the peer mappings cannot be made):
//    ncclAllReduce in place, then the residual kernel.
//
// NCCL is resolved at run time with dlopen: a process that already holds a
// libnccl (torch's) reuses it, so the two never mix.  Only the types come
// from nccl.h.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>
#include <string>
#include <vector>

#include "gemv_core.cuh"

struct reng_model;

namespace reng {
void* tp_handle(reng_model* m);
void tp_set_handle(reng_model* m, void* h);
int tp_rank_of(reng_model* m);
int tp_world_of(reng_model* m);
int tp_device_of(reng_model* m);
uint16_t* tp_x_res(reng_model* m);
float* tp_ss(reng_model* m);
int tp_hidden(reng_model* m);
int* tp_err(reng_model* m);

namespace {
struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    std::string err;
    bool ok = false;
};

NcclApi* api() {
    static NcclApi a;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            a.err = std::string("dlopen libnccl.so.2: ") + dlerror();
            return;
        }
        a.GetUniqueId = (decltype(a.GetUniqueId))dlsym(h, "ncclGetUniqueId");
        a.CommInitRank = (decltype(a.CommInitRank))dlsym(h, "ncclCommInitRank");
        a.AllReduce = (decltype(a.AllReduce))dlsym(h, "ncclAllReduce");
        a.AllGather = (decltype(a.AllGather))dlsym(h, "ncclAllGather");
        a.CommDestroy = (decltype(a.CommDestroy))dlsym(h, "ncclCommDestroy");
        a.GetErrorString = (decltype(a.GetErrorString))dlsym(h, "ncclGetErrorString");
        a.ok = a.GetUniqueId && a.CommInitRank && a.AllReduce && a.AllGather && a.CommDestroy && a.GetErrorString;
        if (!a.ok) a.err = "libnccl.so.2 lacks a symbol";
    });
    return &a;
}

constexpr int kArSlice = 256;    // hidden elements per CTA of the peer all-reduce
constexpr int kArThreads = 64;   // a float4 of the slice per thread

// The peer all-reduce arguments.  Receive area of a rank: [2 parities]
// [W source ranks][kMaxRows][hidden] 64-bit words, each (epoch << 32 |
// f32 bits) of one partial value.  An aligned 8-byte store is single-copy
// atomic, so a receiver that reads the current epoch in a word also reads
// the value stored with it: no fence, no separate flag, and every thread
// waits only for the words of its own elements.
struct ArArgs {
    unsigned long long* recv[kTpMaxWorld];  // every rank's receive area (peer mappings; own at [rank])
    const float* part;             // this rank's partial [M][hidden]
    unsigned* epoch;               // [C] exchanges done per slice (this rank only)
    uint16_t* x_res;               // [M][hidden]
    float* ss;                     // norm partials [M][kSsStride]
    int* err;
    int rank, world, hidden, M;
};

struct TpState {
    ncclComm_t comm = nullptr;
    bool p2p = false;              // the peer all-reduce is set up
    void* region = nullptr;        // this rank's receive area + head key area (exported)
    unsigned* epoch = nullptr;     // [C] all-reduce slices, then the head exchange count
    HeadXchg* hx = nullptr;        // device copy of the head exchange (peer key areas)
    std::vector<void*> mapped;     // peers' regions opened in this process
    ArArgs ar{};
};

size_t ar_recv_words(int world, int hidden) { return (size_t)2 * world * kMaxRows * hidden; }
constexpr size_t kHeadKeyWords = (size_t)2 * kTpMaxWorld * kMaxRows * 2;  // the head key area

__device__ __forceinline__ unsigned long long ar_word(float v, unsigned e) {
    return ((unsigned long long)e << 32) | __float_as_uint(v);
}

__global__ void __launch_bounds__(kArThreads) k_tp_ar_residual(ArArgs a) {
    const int c = blockIdx.x, t = threadIdx.x;
    const int i0 = c * kArSlice + 4 * t;  // this thread's 4 elements (hidden % 16 == 0)
    const bool live = i0 < a.hidden;
    pdl_wait();
    pdl_launch();
    const unsigned e = a.epoch[c] + 1;
    const size_t par = (size_t)(e & 1) * a.world * kMaxRows * a.hidden;
    // 1. push this rank's partial values into every peer's area
    float4 mine[kMaxRows];
#pragma unroll
    for (int m = 0; m < kMaxRows; m++)
        if (m < a.M && live) mine[m] = __ldcg(reinterpret_cast<const float4*>(a.part + (size_t)m * a.hidden + i0));
    if (live)
        for (int r = 0; r < a.world; r++) {
            if (r == a.rank) continue;
            unsigned long long* dst = a.recv[r] + par + (size_t)a.rank * kMaxRows * a.hidden + i0;
#pragma unroll
            for (int m = 0; m < kMaxRows; m++)
                if (m < a.M) {
                    st_words(dst + (size_t)m * a.hidden, ar_word(mine[m].x, e), ar_word(mine[m].y, e));
                    st_words(dst + (size_t)m * a.hidden + 2, ar_word(mine[m].z, e), ar_word(mine[m].w, e));
                }
        }
    // 2. the peers' values of these elements (bounded wait), summed in rank
    //    order; bf16 residual add; norm partials of 16-wide tiles
    const unsigned long long* own = a.recv[a.rank] + par;
    bool late = false;
#pragma unroll
    for (int m = 0; m < kMaxRows; m++) {
        if (m >= a.M) break;
        float sq = 0.f;
        if (live) {
            float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int r = 0; r < a.world; r++) {
                float4 v = mine[m];
                if (r != a.rank) {
                    const unsigned long long* src = own + ((size_t)r * kMaxRows + m) * a.hidden + i0;
                    unsigned long long w0, w1, w2, w3;
                    ld_words(src, w0, w1);
                    ld_words(src + 2, w2, w3);
                    if (((w0 >> 32) != e || (w1 >> 32) != e || (w2 >> 32) != e || (w3 >> 32) != e) && !late) {
                        const unsigned long long t0 = globaltimer();
                        do {
                            ld_words(src, w0, w1);
                            ld_words(src + 2, w2, w3);
                            if (globaltimer() - t0 > kWaitNs) {
                                atomicExch(a.err, RENG_E_TIMEOUT);
                                late = true;
                                break;
                            }
                        } while ((w0 >> 32) != e || (w1 >> 32) != e || (w2 >> 32) != e || (w3 >> 32) != e);
                    }
                    v = make_float4(__uint_as_float((unsigned)w0), __uint_as_float((unsigned)w1),
                                    __uint_as_float((unsigned)w2), __uint_as_float((unsigned)w3));
                }
                if (r == 0) {
                    s = v;
                } else {
                    s.x += v.x;
                    s.y += v.y;
                    s.z += v.z;
                    s.w += v.w;
                }
            }
            uint2* xp = reinterpret_cast<uint2*>(a.x_res + (size_t)m * a.hidden + i0);
            const uint2 x = *xp;
            const float r0 = round_bf16(bf16lo(x.x) + round_bf16(s.x)), r1 = round_bf16(bf16hi(x.x) + round_bf16(s.y));
            const float r2 = round_bf16(bf16lo(x.y) + round_bf16(s.z)), r3 = round_bf16(bf16hi(x.y) + round_bf16(s.w));
            *xp = make_uint2(pack_bf16x2(r0, r1), pack_bf16x2(r2, r3));
            sq = r0 * r0 + r1 * r1 + r2 * r2 + r3 * r3;
        }
        sq += __shfl_xor_sync(0xffffffffu, sq, 1);
        sq += __shfl_xor_sync(0xffffffffu, sq, 2);
        if (live && (t & 3) == 0) a.ss[(size_t)m * kSsStride + i0 / 16] = sq;
    }
    __syncthreads();  // every thread has read this launch's epoch
    if (t == 0) a.epoch[c] = e;
}

// Sets up the peer all-reduce: allocate and export this rank's region,
// all-gather the IPC handles over NCCL, open the peers', and agree (an
// NCCL min over the ranks' outcomes) so every rank takes the same path.
// Returns 1 when set up, 0 (after undoing what it did) when any rank could
// not, -1 when this rank failed after the ranks agreed (the model is then
// not created: the other ranks' exchanges would wait for it in vain).
int ar_setup(reng_model* m, TpState* s, NcclApi* a) {
    const int W = tp_world_of(m), R = tp_rank_of(m), H = tp_hidden(m);
    const char* env = getenv("RENG_TP_P2P");
    if (env && atoi(env) == 0) return 0;  // every rank reads the same environment
    int ok = W <= kTpMaxWorld && H % 16 == 0 ? 1 : 0;
    const size_t words = ar_recv_words(W, H), bytes = (words + kHeadKeyWords) * 8;
    const int C = (H + kArSlice - 1) / kArSlice;
    cudaIpcMemHandle_t mine{};
    if (ok && cudaMalloc(&s->region, bytes) != cudaSuccess) ok = 0;
    if (ok && cudaMemset(s->region, 0, bytes) != cudaSuccess) ok = 0;
    if (ok && cudaMalloc((void**)&s->epoch, (size_t)(C + 1) * 4) != cudaSuccess) ok = 0;
    if (ok && cudaMemset(s->epoch, 0, (size_t)(C + 1) * 4) != cudaSuccess) ok = 0;
    if (ok && cudaMalloc((void**)&s->hx, sizeof(HeadXchg)) != cudaSuccess) ok = 0;
    if (ok && cudaIpcGetMemHandle(&mine, s->region) != cudaSuccess) ok = 0;
    cudaGetLastError();
    // exchange: [W] handles, then the agreement word
    uint8_t* dev = nullptr;
    std::vector<cudaIpcMemHandle_t> all(W);
    int agree = 0;
    if (cudaMalloc((void**)&dev, (size_t)(W + 1) * sizeof(cudaIpcMemHandle_t) + 16) != cudaSuccess) {
        // cannot take part in the exchange the other ranks are entering
        if (s->region) cudaFree(s->region);
        if (s->epoch) cudaFree(s->epoch);
        if (s->hx) cudaFree(s->hx);
        s->region = nullptr;
        s->epoch = nullptr;
        s->hx = nullptr;
        return -1;
    }
    uint8_t* send = dev + (size_t)W * sizeof(cudaIpcMemHandle_t);
    int* okd = reinterpret_cast<int*>(send + sizeof(cudaIpcMemHandle_t));
    bool done = cudaMemcpy(send, &mine, sizeof(mine), cudaMemcpyHostToDevice) == cudaSuccess &&
                a->AllGather(send, dev, sizeof(mine), ncclChar, s->comm, 0) == ncclSuccess &&
                cudaMemcpy(all.data(), dev, (size_t)W * sizeof(mine), cudaMemcpyDeviceToHost) == cudaSuccess;
    s->ar = ArArgs{};
    if (done && ok) {
        for (int r = 0; r < W; r++) {
            if (r == R) {
                s->ar.recv[r] = static_cast<unsigned long long*>(s->region);
                continue;
            }
            void* p = nullptr;
            if (cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                ok = 0;
                break;
            }
            s->mapped.push_back(p);
            s->ar.recv[r] = static_cast<unsigned long long*>(p);
        }
    }
    done = done && cudaMemcpy(okd, &ok, 4, cudaMemcpyHostToDevice) == cudaSuccess &&
           a->AllReduce(okd, okd, 1, ncclInt32, ncclMin, s->comm, 0) == ncclSuccess &&
           cudaMemcpy(&agree, okd, 4, cudaMemcpyDeviceToHost) == cudaSuccess;
    cudaFree(dev);
    if (done && agree == 1) {
        HeadXchg hx{};
        for (int r = 0; r < W; r++) hx.recv[r] = s->ar.recv[r] + words;
        hx.epoch = s->epoch + C;
        hx.rank = R;
        hx.world = W;
        if (cudaMemcpy(s->hx, &hx, sizeof(hx), cudaMemcpyHostToDevice) == cudaSuccess) {
            s->p2p = true;
            s->ar.epoch = s->epoch;
            s->ar.rank = R;
            s->ar.world = W;
            s->ar.hidden = H;
            return 1;
        }
    }
    const int rc = done && agree == 1 ? -1 : 0;  // -1: agreed, then this rank failed
    for (void* p : s->mapped) cudaIpcCloseMemHandle(p);
    s->mapped.clear();
    if (s->region) cudaFree(s->region);
    if (s->epoch) cudaFree(s->epoch);
    if (s->hx) cudaFree(s->hx);
    s->region = nullptr;
    s->epoch = nullptr;
    s->hx = nullptr;
    cudaGetLastError();
    return rc;
}
}  // namespace

int tp_init(reng_model* m, const uint8_t* id) {
    NcclApi* a = api();
    if (!a->ok) return fail(RENG_E_NCCL, a->err);
    ncclUniqueId uid;
    static_assert(sizeof(uid) == 128, "ncclUniqueId is 128 bytes");
    memcpy(&uid, id, sizeof(uid));
    cudaSetDevice(tp_device_of(m));
    TpState* s = new TpState();
    ncclResult_t r = a->CommInitRank(&s->comm, tp_world_of(m), uid, tp_rank_of(m));
    if (r != ncclSuccess) {
        delete s;
        return fail(RENG_E_NCCL, std::string("ncclCommInitRank: ") + a->GetErrorString(r));
    }
    tp_set_handle(m, s);
    if (ar_setup(m, s, a) < 0) return fail(RENG_E_CUDA, "tensor parallel: this rank could not set up the peer exchange");
    return RENG_OK;
}

void tp_destroy(reng_model* m) {
    TpState* s = static_cast<TpState*>(tp_handle(m));
    if (!s) return;
    // every exchange this rank took part in has completed (the caller
    // synchronised its stream): this rank read the epoch of every word a
    // peer stored into its region, and each peer reads every word this rank
    // stored into the peer's region before its own launch ends
    for (void* p : s->mapped) cudaIpcCloseMemHandle(p);
    if (s->region) cudaFree(s->region);
    if (s->epoch) cudaFree(s->epoch);
    if (s->hx) cudaFree(s->hx);
    if (s->comm && api()->ok) api()->CommDestroy(s->comm);
    delete s;
    tp_set_handle(m, nullptr);
}

// 0 no exchange (world 1), 1 NCCL, 2 the peer all-reduce for decode steps.
int tp_exchange_kind(reng_model* m) {
    TpState* s = static_cast<TpState*>(tp_handle(m));
    if (!s) return 0;
    return s->p2p ? 2 : 1;
}

// The device head exchange of a peer-mapped model (null otherwise).
const HeadXchg* tp_head_xchg(reng_model* m) {
    TpState* s = static_cast<TpState*>(tp_handle(m));
    return s && s->p2p ? s->hx : nullptr;
}

bool tp_p2p(reng_model* m, int M) {
    TpState* s = static_cast<TpState*>(tp_handle(m));
    return s && s->p2p && M <= kMaxRows;
}

cudaError_t tp_allreduce(reng_model* m, float* buf, size_t count, cudaStream_t st) {
    NcclApi* a = api();
    TpState* s = static_cast<TpState*>(tp_handle(m));
    if (!a->ok || !s) return cudaErrorNotReady;
    ncclResult_t r = a->AllReduce(buf, buf, count, ncclFloat32, ncclSum, s->comm, st);
    if (r != ncclSuccess) {
        set_error(std::string("ncclAllReduce: ") + a->GetErrorString(r));
        return cudaErrorUnknown;
    }
    return cudaSuccess;
}

// The peer all-reduce + residual of M <= kMaxRows rows of partials.
cudaError_t launch_tp_ar_residual(reng_model* m, const float* part, int M, cudaStream_t st) {
    TpState* s = static_cast<TpState*>(tp_handle(m));
    if (!s || !s->p2p || M < 1 || M > kMaxRows) return cudaErrorInvalidValue;
    ArArgs a = s->ar;
    a.part = part;
    a.x_res = tp_x_res(m);
    a.ss = tp_ss(m);
    a.err = tp_err(m);
    a.M = M;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3((unsigned)((a.hidden + kArSlice - 1) / kArSlice));
    cfg.blockDim = dim3(kArThreads);
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_tp_ar_residual, a);
}

// x_res = bf16(x_res + bf16(partial)) (tp.rs:17-21: f32 partials reduced in
// f32, cast to bf16, residual-added in bf16) and the norm partials of x_res.
__global__ void __launch_bounds__(256) k_tp_residual(uint16_t* x_res, const float* part, float* ss,
                                                     int hidden) {
    const int m = blockIdx.x;
    pdl_wait();
    pdl_launch();
    const int nv = hidden / 8;
    for (int base = 0; base < nv; base += blockDim.x) {
        const int i = base + threadIdx.x;
        float s = 0.f;
        if (i < nv) {
            uint4* xp = reinterpret_cast<uint4*>(x_res + (size_t)m * hidden) + i;
            const float4* pp = reinterpret_cast<const float4*>(part + (size_t)m * hidden) + 2 * i;
            uint4 x = *xp;
            float4 p0 = pp[0], p1 = pp[1];
            float r[8] = {round_bf16(bf16lo(x.x) + round_bf16(p0.x)), round_bf16(bf16hi(x.x) + round_bf16(p0.y)),
                          round_bf16(bf16lo(x.y) + round_bf16(p0.z)), round_bf16(bf16hi(x.y) + round_bf16(p0.w)),
                          round_bf16(bf16lo(x.z) + round_bf16(p1.x)), round_bf16(bf16hi(x.z) + round_bf16(p1.y)),
                          round_bf16(bf16lo(x.w) + round_bf16(p1.z)), round_bf16(bf16hi(x.w) + round_bf16(p1.w))};
#pragma unroll
            for (int e = 0; e < 8; e++) s += r[e] * r[e];
            uint4 o;
            o.x = pack_bf16x2(r[0], r[1]);
            o.y = pack_bf16x2(r[2], r[3]);
            o.z = pack_bf16x2(r[4], r[5]);
            o.w = pack_bf16x2(r[6], r[7]);
            *xp = o;
        }
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        if (i < nv && (i & 1) == 0) ss[(size_t)m * kSsStride + (i >> 1)] = s;
    }
}

cudaError_t launch_tp_residual(reng_model* m, const float* part, int M, bool pdl, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(M);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_tp_residual, tp_x_res(m), part, tp_ss(m), tp_hidden(m));
}

}  // namespace reng

// The failure path of the peer exchange on one GPU: the exchange kernel as
// rank 0 of a two-rank group whose rank 1 never runs, so the epoch words it
// waits for are never written.  Every wait gives up after its bound, the
// kernel records RENG_E_TIMEOUT and returns; the context must stay usable.
extern "C" int reng_tp_peer_wait_check(int device) {
    using namespace reng;
    RENG_CUDA_TRY(cudaSetDevice(device));
    constexpr int H = 512, M = 1;
    const size_t words = ar_recv_words(2, H);
    unsigned long long *mine = nullptr, *peer = nullptr;
    unsigned* epoch = nullptr;
    float *part = nullptr, *ss = nullptr;
    uint16_t* x = nullptr;
    int* err = nullptr;
    int rc = RENG_OK;
    auto alloc = [&](void** p, size_t b) {
        if (rc == RENG_OK && cudaMalloc(p, b) != cudaSuccess) rc = fail(RENG_E_NOMEM, "reng_tp_peer_wait_check: cudaMalloc");
        if (rc == RENG_OK) cudaMemset(*p, 0, b);
    };
    alloc((void**)&mine, words * 8);
    alloc((void**)&peer, words * 8);
    alloc((void**)&epoch, 64);
    alloc((void**)&part, (size_t)M * H * 4);
    alloc((void**)&ss, (size_t)M * kSsStride * 4);
    alloc((void**)&x, (size_t)M * H * 2);
    alloc((void**)&err, 4);
    if (rc == RENG_OK) {
        ArArgs a{};
        a.recv[0] = mine;  // rank 0: this launch
        a.recv[1] = peer;  // rank 1: receives this rank's values, never answers
        a.part = part;
        a.epoch = epoch;
        a.x_res = x;
        a.ss = ss;
        a.err = err;
        a.rank = 0;
        a.world = 2;
        a.hidden = H;
        a.M = M;
        k_tp_ar_residual<<<(H + kArSlice - 1) / kArSlice, kArThreads>>>(a);
        int h = 0;
        if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpy(&h, err, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
            rc = fail(RENG_E_CUDA, std::string("reng_tp_peer_wait_check: ") + cudaGetErrorString(cudaGetLastError()));
        else if (h == RENG_E_TIMEOUT)
            rc = fail(RENG_E_TIMEOUT, "reng_tp_peer_wait_check: the exchange gave up on its bounded wait (expected)");
        else
            rc = fail(RENG_E_STATE, "reng_tp_peer_wait_check: the exchange did not report the missing peer");
    }
    for (void* p : {(void*)mine, (void*)peer, (void*)epoch, (void*)part, (void*)ss, (void*)x, (void*)err})
        if (p) cudaFree(p);
    return rc;
}

extern "C" int reng_tp_unique_id(uint8_t out[128]) {
    RENG_CHECK_ARG(out != nullptr, "reng_tp_unique_id: out is NULL");
    reng::NcclApi* a = reng::api();
    if (!a->ok) return reng::fail(RENG_E_NCCL, a->err);
    ncclUniqueId uid;
    ncclResult_t r = a->GetUniqueId(&uid);
    if (r != ncclSuccess) return reng::fail(RENG_E_NCCL, std::string("ncclGetUniqueId: ") + a->GetErrorString(r));
    memcpy(out, &uid, 128);
    return RENG_OK;
}
