// FP8 weight quantizer on the device: the reference's reng_fp8::quantize_with
// (crates/reng-fp8/src/lib.rs:519-563) with its encode (lib.rs:154-201).
//
// One CTA per matrix row.  The row is loaded once into registers with
// 16-byte streaming loads, its absmax is reduced across the CTA, the scale
// is formed with the reference's f32 arithmetic (absmax / (max_finite *
// backoff), IEEE division), and every element is encoded from the
// registers: HBM traffic is the algorithmic 2 B read + 1 B written per
// element + 4 B per row.
//
// Encoding uses the hardware RNE converters.  Equality with the
// reference's integer encoder holds for every f32 input:
//  * E4M3: the reference's format shares bias 7, subnormals and every
//    finite code up to 240 with OCP E4M3 (the cvt target); above 240 the
//    reference saturates to 240 (0x77) where OCP continues to 448.  Every
//    |x| >= 240 encodes to 0x77 in the reference (240 < |x| < 248 rounds to
//    240; |x| >= 248 rounds to 256, which saturates), so clamping to
//    +-240 before the cvt gives the same byte.
//  * E5M2: both saturate at 57344 (0x7b) under .satfinite.
//  * NaN: the reference writes sign|0x7f; set explicitly.  A NaN the
//    division itself generates (+-inf / inf, when an infinite weight makes
//    the row scale infinite) takes the sign of the x86 default NaN (the
//    "real indefinite", sign bit set), the platform the reference runs on;
//    a NaN weight keeps its own sign.
//  * f32 subnormals and zeros encode to the signed zero in both.
// tests/test_fp8_gpu.py checks this claim over all 2^32 f32 inputs.
#include <algorithm>
#include <cmath>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "fp8_product.h"

namespace reng {

// Two f32 -> two E4M3 codes (first argument in the low byte).
__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}
__device__ __forceinline__ uint32_t cvt_e5m2x2(float lo, float hi) {
    uint16_t r;
    asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}

template <int FMT>
__device__ __forceinline__ uint32_t encode2(float a, float b) {
    uint32_t c;
    if (FMT == RENG_FP8_E4M3) {
        c = cvt_e4m3x2(fminf(fmaxf(a, -240.0f), 240.0f), fminf(fmaxf(b, -240.0f), 240.0f));
    } else {
        c = cvt_e5m2x2(a, b);
    }
    if (isnan(a)) c = (c & 0xff00u) | ((__float_as_uint(a) >> 24) & 0x80u) | 0x7fu;
    if (isnan(b)) c = (c & 0x00ffu) | ((((__float_as_uint(b) >> 24) & 0x80u) | 0x7fu) << 8);
    return c;
}

// x / s as the reference's host computes it: IEEE division; a NaN weight
// comes through as itself, sign included (x86 returns the NaN operand; GPU
// arithmetic would return its canonical positive NaN), and a NaN generated
// by the division is x86's default NaN, whose sign bit is set.
__device__ __forceinline__ float div_host(float x, float s) {
    if (isnan(x)) return x;
    float q = __fdiv_rn(x, s);
    if (isnan(q)) q = __uint_as_float(0xffc00000u);
    return q;
}

// The same quotient without the division (fp8_product.h: Markstein's
// correction of x * RN(1 / s)), for rows fp8_product_ok admits.
template <int FMT>
__device__ __forceinline__ uint2 encode8_product(uint4 v, float s, float r) {
    uint2 o;
    uint32_t c0 = encode2<FMT>(fp_quotient(bf16lo(v.x), s, r), fp_quotient(bf16hi(v.x), s, r));
    uint32_t c1 = encode2<FMT>(fp_quotient(bf16lo(v.y), s, r), fp_quotient(bf16hi(v.y), s, r));
    uint32_t c2 = encode2<FMT>(fp_quotient(bf16lo(v.z), s, r), fp_quotient(bf16hi(v.z), s, r));
    uint32_t c3 = encode2<FMT>(fp_quotient(bf16lo(v.w), s, r), fp_quotient(bf16hi(v.w), s, r));
    o.x = c0 | (c1 << 16);
    o.y = c2 | (c3 << 16);
    return o;
}

// 8 bf16 (one uint4) / s -> 8 codes (one uint2).
template <int FMT>
__device__ __forceinline__ uint2 encode8(uint4 v, float s) {
    uint2 o;
    uint32_t c0 = encode2<FMT>(div_host(bf16lo(v.x), s), div_host(bf16hi(v.x), s));
    uint32_t c1 = encode2<FMT>(div_host(bf16lo(v.y), s), div_host(bf16hi(v.y), s));
    uint32_t c2 = encode2<FMT>(div_host(bf16lo(v.z), s), div_host(bf16hi(v.z), s));
    uint32_t c3 = encode2<FMT>(div_host(bf16lo(v.w), s), div_host(bf16hi(v.w), s));
    o.x = c0 | (c1 << 16);
    o.y = c2 | (c3 << 16);
    return o;
}

__device__ __forceinline__ float absmax8(uint4 v, float m) {
    // '>' against the running value, as the reference does (NaN ignored).
    float t[8] = {bf16lo(v.x), bf16hi(v.x), bf16lo(v.y), bf16hi(v.y),
                  bf16lo(v.z), bf16hi(v.z), bf16lo(v.w), bf16hi(v.w)};
#pragma unroll
    for (int i = 0; i < 8; i++) {
        float a = fabsf(t[i]);
        if (a > m) m = a;
    }
    return m;
}

__device__ __forceinline__ float block_max(float v, float* red) {
    v = warp_max(v);
    int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) red[w] = v;
    __syncthreads();
    if (w == 0) {
        float x = (l < (int)(blockDim.x >> 5)) ? red[l] : 0.0f;
        x = warp_max(x);
        if (l == 0) red[32] = x;
    }
    __syncthreads();
    float r = red[32];
    __syncthreads();
    return r;
}

enum { MODE_FUSED_PCS = 0, MODE_FUSED_UNIT = 1, MODE_ABSMAX = 2, MODE_ENCODE = 3 };

// Vector path: cols % 8 == 0, 16-byte aligned rows.  R = uint4 chunks per
// thread held in registers (row length <= R * 8 * blockDim).
template <int FMT, int R>
__global__ void __launch_bounds__(256) k_fp8_rows_vec(const uint16_t* __restrict__ w,
                                                      int64_t rows, int64_t cols, int mode,
                                                      float full, uint8_t* __restrict__ codes,
                                                      float* __restrict__ scales, int product) {
    __shared__ float red[33];
    const int nch = (int)(cols >> 3);
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const uint4* src = reinterpret_cast<const uint4*>(w + row * cols);
        uint4 v[R];
        float m = 0.0f;
#pragma unroll
        for (int r = 0; r < R; r++) {
            int c = threadIdx.x + r * blockDim.x;
            if (c < nch) {
                v[r] = ldg_stream(src + c);
                m = absmax8(v[r], m);
            }
        }
        float s;
        if (mode == MODE_ENCODE) {
            s = scales[row];
        } else if (mode == MODE_FUSED_UNIT) {
            s = 1.0f;
            if (threadIdx.x == 0) scales[row] = s;
        } else {
            m = block_max(m, red);
            if (mode == MODE_ABSMAX) {
                if (threadIdx.x == 0) scales[row] = m;
                continue;
            }
            s = m > 0.0f ? __fdiv_rn(m, full) : 1.0f;
            if (threadIdx.x == 0) scales[row] = s;
        }
        uint2* dst = reinterpret_cast<uint2*>(codes + row * cols);
        // m bounds this thread's weights (its own absmax, or the row's)
        const float rq = __frcp_rn(s);
        if (product && fp8_product_ok(s, rq, m)) {
#pragma unroll
            for (int r = 0; r < R; r++) {
                int c = threadIdx.x + r * blockDim.x;
                if (c < nch) dst[c] = encode8_product<FMT>(v[r], s, rq);
            }
        } else {
#pragma unroll
            for (int r = 0; r < R; r++) {
                int c = threadIdx.x + r * blockDim.x;
                if (c < nch) dst[c] = encode8<FMT>(v[r], s);
            }
        }
    }
}

// Generic path (any cols, any alignment): two passes over the row.
template <int FMT>
__global__ void __launch_bounds__(256) k_fp8_rows_any(const uint16_t* __restrict__ w,
                                                      int64_t rows, int64_t cols, int mode,
                                                      float full, uint8_t* __restrict__ codes,
                                                      float* __restrict__ scales) {
    __shared__ float red[33];
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const uint16_t* src = w + row * cols;
        float s;
        if (mode == MODE_ENCODE) {
            s = scales[row];
        } else if (mode == MODE_FUSED_UNIT) {
            s = 1.0f;
            if (threadIdx.x == 0) scales[row] = s;
        } else {
            float m = 0.0f;
            for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
                float a = fabsf(bf16_bits_to_f32(src[c]));
                if (a > m) m = a;
            }
            m = block_max(m, red);
            if (mode == MODE_ABSMAX) {
                if (threadIdx.x == 0) scales[row] = m;
                continue;
            }
            s = m > 0.0f ? __fdiv_rn(m, full) : 1.0f;
            if (threadIdx.x == 0) scales[row] = s;
        }
        for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
            float x = div_host(bf16_bits_to_f32(src[c]), s);
            codes[row * cols + c] = (uint8_t)(encode2<FMT>(x, 0.0f) & 0xffu);
        }
    }
}

// HwExpBias: the tensor absmax over the row absmaxes (already in scales),
// then the exponent bias choice of reng_fp8::choose_exp_bias
// (lib.rs:464-475) and the power-of-two scale written to every row.
__device__ __forceinline__ float pow2_exact(int e) {
    return e >= -126 ? __uint_as_float((uint32_t)(e + 127) << 23) : __uint_as_float(1u << (e + 149));
}

template <int FMT>
__global__ void __launch_bounds__(1024) k_fp8_hw_choose(float* scales, int64_t rows, float backoff,
                                                        uint32_t* bias_out) {
    __shared__ float red[33];
    __shared__ float s_scale;
    float m = 0.0f;
    for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) m = fmaxf(m, scales[r]);
    m = block_max(m, red);
    if (threadIdx.x == 0) {
        const int def = FMT == RENG_FP8_E4M3 ? 7 : 15;
        const float maxf = FMT == RENG_FP8_E4M3 ? 240.0f : 57344.0f;
        const uint32_t e4[4] = {15, 11, 7, 3};
        const int nb = FMT == RENG_FP8_E4M3 ? 4 : 1;
        float a = __fdiv_rn(m, backoff);
        uint32_t b = FMT == RENG_FP8_E4M3 ? 3u : 15u;
        for (int i = 0; i < nb; i++) {
            uint32_t cand = FMT == RENG_FP8_E4M3 ? e4[i] : 15u;
            if (a <= maxf * pow2_exact(def - (int)cand)) {
                b = cand;
                break;
            }
        }
        *bias_out = b;
        s_scale = pow2_exact(def - (int)b);
    }
    __syncthreads();
    float s = s_scale;
    for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) scales[r] = s;
}

template <int FMT>
__global__ void k_fp8_encode_flat(const float* __restrict__ x, int64_t n, uint8_t* __restrict__ c) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        c[i] = (uint8_t)(encode2<FMT>(x[i], 0.0f) & 0xffu);
}

// reng_fp8::decode (lib.rs:205-225).
__device__ __forceinline__ float fp8_decode_dev(uint32_t code, int fmt) {
    const int mb = fmt == RENG_FP8_E4M3 ? 3 : 2;
    const int bias = fmt == RENG_FP8_E4M3 ? 7 : 15;
    const int eb = 7 - mb;
    float sign = (code & 0x80u) ? -1.0f : 1.0f;
    uint32_t mant = code & ((1u << mb) - 1u);
    uint32_t ef = (code & 0x7fu) >> mb;
    if (ef == (1u << eb) - 1u) return mant == 0 ? sign * __int_as_float(0x7f800000) : __int_as_float(0x7fc00000);
    float frac = (float)mant / (float)(1u << mb);
    if (ef == 0) return sign * frac * pow2_exact(1 - bias);
    return sign * (1.0f + frac) * pow2_exact((int)ef - bias);
}

__global__ void k_fp8_decode_flat(const uint8_t* __restrict__ c, int64_t n, int fmt,
                                  float* __restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = fp8_decode_dev(c[i], fmt);
}

// ------------------------------------------------------------ launcher --
template <int FMT>
static void launch_rows(const uint16_t* w, int64_t rows, int64_t cols, int mode, float full,
                        uint8_t* codes, float* scales, bool vec, cudaStream_t st) {
    int grid = (int)std::min<int64_t>(rows, 148 * 64);
    // The division-free quotient (bit-identical to the division; B200,
    // config-0 matrix over a 16-matrix rotation: 23.3 -> 20.1 us, 2.16 ->
    // 2.50 TB/s) unless RENG_FP8_PRODUCT=0 asks for the IEEE division
    const char* pe = getenv("RENG_FP8_PRODUCT");
    const int product = pe && atoi(pe) == 0 ? 0 : 1;
    if (!vec) {
        k_fp8_rows_any<FMT><<<grid, 256, 0, st>>>(w, rows, cols, mode, full, codes, scales);
        return;
    }
    int64_t nch = cols / 8;
    if (nch <= 256)
        k_fp8_rows_vec<FMT, 1><<<grid, 256, 0, st>>>(w, rows, cols, mode, full, codes, scales, product);
    else if (nch <= 512)
        k_fp8_rows_vec<FMT, 2><<<grid, 256, 0, st>>>(w, rows, cols, mode, full, codes, scales, product);
    else if (nch <= 1024)
        k_fp8_rows_vec<FMT, 4><<<grid, 256, 0, st>>>(w, rows, cols, mode, full, codes, scales, product);
    else if (nch <= 2048)
        k_fp8_rows_vec<FMT, 8><<<grid, 256, 0, st>>>(w, rows, cols, mode, full, codes, scales, product);
    else
        k_fp8_rows_any<FMT><<<grid, 256, 0, st>>>(w, rows, cols, mode, full, codes, scales);
}

// Device-pointer quantizer used by the C ABI and by the model's fp8 load
// path.  bias_dev is a device u32 used only by the HwExpBias scheme.
int fp8_quantize_device(const uint16_t* w, int64_t rows, int64_t cols, int fmt, int scaling,
                        float backoff, uint8_t* codes, float* scales, uint32_t* bias_dev,
                        cudaStream_t st) {
    bool vec = (cols % 8 == 0) && ((uintptr_t)w % 16 == 0) && ((uintptr_t)codes % 8 == 0);
    float full = (fmt == RENG_FP8_E4M3 ? 240.0f : 57344.0f) * backoff;
    auto run = [&](int mode) {
        if (fmt == RENG_FP8_E4M3)
            launch_rows<RENG_FP8_E4M3>(w, rows, cols, mode, full, codes, scales, vec, st);
        else
            launch_rows<RENG_FP8_E5M2>(w, rows, cols, mode, full, codes, scales, vec, st);
    };
    if (scaling == RENG_SCALING_PCS) {
        run(MODE_FUSED_PCS);
    } else if (scaling == RENG_SCALING_UNIT) {
        run(MODE_FUSED_UNIT);
    } else {
        run(MODE_ABSMAX);
        if (fmt == RENG_FP8_E4M3)
            k_fp8_hw_choose<RENG_FP8_E4M3><<<1, 1024, 0, st>>>(scales, rows, backoff, bias_dev);
        else
            k_fp8_hw_choose<RENG_FP8_E5M2><<<1, 1024, 0, st>>>(scales, rows, backoff, bias_dev);
        run(MODE_ENCODE);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(RENG_E_CUDA, std::string("fp8 quantize launch: ") + cudaGetErrorString(e));
    return RENG_OK;
}

}  // namespace reng

using namespace reng;

// The argument checks of both quantize entry points; `who` names the entry
// the caller used, so reng_last_error() reports that one.
static int check_quant_args(const char* who, const uint16_t* w, int64_t rows, int64_t cols, int fmt,
                            int scaling, float backoff, uint8_t* codes, float* scales, uint32_t* exp_bias,
                            int mem) {
    const std::string f = std::string(who) + ": ";
    RENG_CHECK_ARG(rows > 0 && cols > 0, f + "empty shape " + std::to_string(rows) + " x " + std::to_string(cols));
    RENG_CHECK_ARG(backoff > 0.0f && std::isfinite(backoff),
                   f + "backoff " + std::to_string(backoff) + " is not positive and finite");
    RENG_CHECK_ARG(fmt == RENG_FP8_E4M3 || fmt == RENG_FP8_E5M2, f + "unknown format");
    RENG_CHECK_ARG(scaling >= RENG_SCALING_PCS && scaling <= RENG_SCALING_UNIT, f + "unknown scaling");
    RENG_CHECK_ARG(w && codes && scales && exp_bias, f + "NULL buffer");
    RENG_CHECK_ARG(mem == RENG_MEM_DEVICE || mem == RENG_MEM_HOST, f + "bad mem");
    RENG_CHECK_ARG(rows <= (int64_t)1 << 40 && cols <= (int64_t)1 << 40 && rows <= ((int64_t)1 << 62) / cols,
                   f + "shape overflows");
    return RENG_OK;
}

extern "C" int reng_fp8_quantize(const uint16_t* w, int64_t rows, int64_t cols, int fmt,
                                 int scaling, float backoff, uint8_t* codes, float* scales,
                                 uint32_t* exp_bias, int mem, void* stream) {
    int rc = check_quant_args("reng_fp8_quantize", w, rows, cols, fmt, scaling, backoff, codes, scales,
                              exp_bias, mem);
    if (rc) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    const size_t nel = (size_t)rows * (size_t)cols;
    const uint32_t def_bias = fmt == RENG_FP8_E4M3 ? 7u : 15u;
    uint16_t* dw = const_cast<uint16_t*>(w);
    uint8_t* dc = codes;
    float* ds = scales;
    uint32_t* dbias = nullptr;
    bool host = mem == RENG_MEM_HOST;
    // One allocation holds the device copies (host mode) and the bias word.
    size_t off_c = host ? nel * 2 : 0;
    size_t off_s = host ? ((off_c + nel + 255) / 256) * 256 : 0;
    size_t off_b = host ? off_s + (((size_t)rows * 4 + 255) / 256) * 256 : 0;
    size_t bytes = off_b + 256;
    char* buf = nullptr;
    const bool need_buf = host || scaling == RENG_SCALING_HW;
    if (need_buf) {
        RENG_CUDA_TRY(cudaMallocAsync((void**)&buf, bytes, st));
        dbias = reinterpret_cast<uint32_t*>(buf + off_b);
    }
    if (host) {
        dw = reinterpret_cast<uint16_t*>(buf);
        dc = reinterpret_cast<uint8_t*>(buf + off_c);
        ds = reinterpret_cast<float*>(buf + off_s);
        rc = cudaMemcpyAsync(dw, w, nel * 2, cudaMemcpyHostToDevice, st) == cudaSuccess ? 0 : -1;
        if (rc) {
            cudaFreeAsync(buf, st);
            return fail(RENG_E_CUDA, "reng_fp8_quantize: upload failed");
        }
    }
    rc = fp8_quantize_device(dw, rows, cols, fmt, scaling, backoff, dc, ds, dbias, st);
    if (rc == RENG_OK) {
        uint32_t b = def_bias;
        cudaError_t e = cudaSuccess;
        if (host) {
            e = cudaMemcpyAsync(codes, dc, nel, cudaMemcpyDeviceToHost, st);
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(scales, ds, (size_t)rows * 4, cudaMemcpyDeviceToHost, st);
        }
        if (e == cudaSuccess && scaling == RENG_SCALING_HW)
            e = cudaMemcpyAsync(&b, dbias, 4, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess && (host || scaling == RENG_SCALING_HW)) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) rc = fail(RENG_E_CUDA, std::string("reng_fp8_quantize: ") + cudaGetErrorString(e));
        else *exp_bias = b;
    }
    if (need_buf) cudaFreeAsync(buf, st);
    return rc;
}

extern "C" int reng_fp8_encode(const float* x, int64_t n, int fmt, uint8_t* codes, void* stream) {
    RENG_CHECK_ARG(n >= 0 && (n == 0 || (x && codes)), "reng_fp8_encode: bad buffers");
    RENG_CHECK_ARG(fmt == RENG_FP8_E4M3 || fmt == RENG_FP8_E5M2, "reng_fp8_encode: unknown format");
    if (n == 0) return RENG_OK;
    cudaStream_t st = (cudaStream_t)stream;
    int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 32);
    if (fmt == RENG_FP8_E4M3) k_fp8_encode_flat<RENG_FP8_E4M3><<<grid, 256, 0, st>>>(x, n, codes);
    else k_fp8_encode_flat<RENG_FP8_E5M2><<<grid, 256, 0, st>>>(x, n, codes);
    RENG_CUDA_TRY(cudaGetLastError());
    return RENG_OK;
}

extern "C" int reng_fp8_decode(const uint8_t* codes, int64_t n, int fmt, float* out, void* stream) {
    RENG_CHECK_ARG(n >= 0 && (n == 0 || (codes && out)), "reng_fp8_decode: bad buffers");
    RENG_CHECK_ARG(fmt == RENG_FP8_E4M3 || fmt == RENG_FP8_E5M2, "reng_fp8_decode: unknown format");
    if (n == 0) return RENG_OK;
    cudaStream_t st = (cudaStream_t)stream;
    int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 32);
    k_fp8_decode_flat<<<grid, 256, 0, st>>>(codes, n, fmt, out);
    RENG_CUDA_TRY(cudaGetLastError());
    return RENG_OK;
}

// ------------------------------------------------- allocation-free variant --
// reng_fp8_quantize with host buffers stages the matrix, the codes, the
// scales and the exponent-bias word in device memory it allocates per call.
// This variant stages them in one fixed array of device memory instead, so
// it never enters the CUDA allocator.  The array is a file-scope __device__
// object: every GPU that loads this library holds its 6.25 MiB until the
// process exits, and every call on a device shares it.
namespace {
constexpr int64_t kNoAllocMaxElems = (int64_t)1 << 21;  // 2,097,152 weights (4 MiB of bf16)
constexpr int64_t kNoAllocMaxRows = (int64_t)1 << 16;   // 65,536 rows
constexpr size_t kNoAllocOffCodes = (size_t)kNoAllocMaxElems * 2;
constexpr size_t kNoAllocOffScales = kNoAllocOffCodes + (size_t)kNoAllocMaxElems;
constexpr size_t kNoAllocOffBias = kNoAllocOffScales + (size_t)kNoAllocMaxRows * 4;
constexpr size_t kNoAllocBytes = kNoAllocOffBias + 256;

static __device__ __align__(256) unsigned char g_fp8_noalloc_scratch[kNoAllocBytes];

// The array's device address, looked up once per device.  In host code the
// symbol itself is only a host-side stand-in; a kernel given it would read
// the wrong memory, so only this address is ever passed on.
std::mutex g_noalloc_mu;
std::vector<unsigned char*> g_noalloc_addr;

int noalloc_scratch(int device, unsigned char** out) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if ((int)g_noalloc_addr.size() <= device) g_noalloc_addr.resize(device + 1, nullptr);
    if (g_noalloc_addr[device] == nullptr) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_fp8_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr)
            return fail(RENG_E_CUDA, std::string("reng_fp8_quantize_noalloc: cudaGetSymbolAddress: ") +
                                         cudaGetErrorString(e));
        g_noalloc_addr[device] = static_cast<unsigned char*>(p);
    }
    *out = g_noalloc_addr[device];
    return RENG_OK;
}
}  // namespace

extern "C" int reng_fp8_quantize_noalloc(const uint16_t* w, int64_t rows, int64_t cols, int fmt,
                                         int scaling, float backoff, uint8_t* codes, float* scales,
                                         uint32_t* exp_bias, void* stream) {
    int rc = check_quant_args("reng_fp8_quantize_noalloc", w, rows, cols, fmt, scaling, backoff, codes,
                              scales, exp_bias, RENG_MEM_HOST);
    if (rc) return rc;
    if (rows > kNoAllocMaxRows || rows * cols > kNoAllocMaxElems)
        return fail(RENG_E_INVAL, "reng_fp8_quantize_noalloc: " + std::to_string(rows) + " x " +
                                      std::to_string(cols) + " exceeds the fixed scratch (at most " +
                                      std::to_string(kNoAllocMaxRows) + " rows and " +
                                      std::to_string(kNoAllocMaxElems) + " elements)");
    int device = 0;
    RENG_CUDA_TRY(cudaGetDevice(&device));
    unsigned char* base = nullptr;
    rc = noalloc_scratch(device, &base);
    if (rc) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    const size_t nel = (size_t)rows * (size_t)cols;
    uint16_t* dw = reinterpret_cast<uint16_t*>(base);
    uint8_t* dc = base + kNoAllocOffCodes;
    float* ds = reinterpret_cast<float*>(base + kNoAllocOffScales);
    uint32_t* db = reinterpret_cast<uint32_t*>(base + kNoAllocOffBias);
    // Nothing in the array has to start at zero: the absmax, scale and bias
    // of this call overwrite whatever the previous call left there.
    RENG_CUDA_TRY(cudaMemcpyAsync(dw, w, nel * 2, cudaMemcpyHostToDevice, st));
    rc = fp8_quantize_device(dw, rows, cols, fmt, scaling, backoff, dc, ds, db, st);
    if (rc) return rc;
    uint32_t b = fmt == RENG_FP8_E4M3 ? 7u : 15u;
    RENG_CUDA_TRY(cudaMemcpyAsync(codes, dc, nel, cudaMemcpyDeviceToHost, st));
    RENG_CUDA_TRY(cudaMemcpyAsync(scales, ds, (size_t)rows * 4, cudaMemcpyDeviceToHost, st));
    if (scaling == RENG_SCALING_HW) RENG_CUDA_TRY(cudaMemcpyAsync(&b, db, 4, cudaMemcpyDeviceToHost, st));
    RENG_CUDA_TRY(cudaStreamSynchronize(st));
    *exp_bias = b;
    return RENG_OK;
}
