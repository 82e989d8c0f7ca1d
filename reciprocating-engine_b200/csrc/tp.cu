// Tensor parallelism: the NCCL communicator of a model and the all-reduce of
// the f32 o_proj / down_proj partials after each half-layer (the reference's
// TpModel, crates/reng-synapse/src/tp.rs:1-42 and :709-793, with its HCCL
// all-reduce, hccl.rs:477-506 / :646-651).
//
// NCCL is resolved at run time with dlopen: a process that already holds a
// libnccl (torch's) reuses it, so the two never mix.  Only the types come
// from nccl.h.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>
#include <string>

#include "decode.cuh"

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

namespace {
struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
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
        a.CommDestroy = (decltype(a.CommDestroy))dlsym(h, "ncclCommDestroy");
        a.GetErrorString = (decltype(a.GetErrorString))dlsym(h, "ncclGetErrorString");
        a.ok = a.GetUniqueId && a.CommInitRank && a.AllReduce && a.CommDestroy && a.GetErrorString;
        if (!a.ok) a.err = "libnccl.so.2 lacks a symbol";
    });
    return &a;
}
}  // namespace

int tp_init(reng_model* m, const uint8_t* id) {
    NcclApi* a = api();
    if (!a->ok) return fail(RENG_E_NCCL, a->err);
    ncclUniqueId uid;
    static_assert(sizeof(uid) == 128, "ncclUniqueId is 128 bytes");
    memcpy(&uid, id, sizeof(uid));
    ncclComm_t comm = nullptr;
    cudaSetDevice(tp_device_of(m));
    ncclResult_t r = a->CommInitRank(&comm, tp_world_of(m), uid, tp_rank_of(m));
    if (r != ncclSuccess) return fail(RENG_E_NCCL, std::string("ncclCommInitRank: ") + a->GetErrorString(r));
    tp_set_handle(m, comm);
    return RENG_OK;
}

void tp_destroy(reng_model* m) {
    void* h = tp_handle(m);
    if (h && api()->ok) api()->CommDestroy((ncclComm_t)h);
    tp_set_handle(m, nullptr);
}

cudaError_t tp_allreduce(reng_model* m, float* buf, size_t count, cudaStream_t st) {
    NcclApi* a = api();
    if (!a->ok || !tp_handle(m)) return cudaErrorNotReady;
    ncclResult_t r = a->AllReduce(buf, buf, count, ncclFloat32, ncclSum, (ncclComm_t)tp_handle(m), st);
    if (r != ncclSuccess) {
        set_error(std::string("ncclAllReduce: ") + a->GetErrorString(r));
        return cudaErrorUnknown;
    }
    return cudaSuccess;
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
        if (i < nv && (i & 1) == 0) ss[(i >> 1) * kRowsCap + m] = s;
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
