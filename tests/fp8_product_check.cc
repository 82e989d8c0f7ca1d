// CPU check of the quantizer's division-free quotient
// (reciprocating-engine_b200/csrc/fp8_product.h) against IEEE division, and
// of the FP8 codes through the C restatement's encoder (oracle/fp8_oracle.c,
// the reference's reng_fp8::encode).
//
//   fp8_product_check <absmax stride> <backoff> [<backoff> ...]
//
// For every stride-th positive finite bf16 absmax m and every backoff b, the
// scale is s = m / (max_finite * b) as the reference forms it (E4M3 and E5M2
// maxima), r = 1 / s.  For each of the 65536 bf16 weights x the product path
// admits (fp8_product_ok with xmax = |x|): the quotient's bits must equal
// x / s wherever |x| >= 2^-102 and |x / s| >= 2^-126, its sign must be x's,
// and its E4M3 and
// E5M2 codes must equal those of x / s everywhere (NaN weights: the encoder's
// sign | 0x7f on both sides).  Prints one line per format and exits 1 on any
// difference.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "fp8_product.h"

extern "C" uint8_t orc_fp8_encode(float x, int fmt);

static float bf16(uint32_t b) {
    uint32_t u = b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

int main(int argc, char** argv) {
    if (argc < 3) {
        fprintf(stderr, "usage: %s <absmax stride> <backoff>...\n", argv[0]);
        return 2;
    }
    const int stride = atoi(argv[1]);
    std::vector<float> backoffs;
    for (int i = 2; i < argc; i++) backoffs.push_back((float)atof(argv[i]));
    long long bad_total = 0;
    for (int fmt = 0; fmt < 2; fmt++) {
        const float maxf = fmt == 0 ? 240.0f : 57344.0f;
        long long rows = 0, checked = 0, refused = 0, bits_bad = 0, code_bad = 0, sub = 0;
        for (float bo : backoffs) {
            const float full = maxf * bo;
#pragma omp parallel for schedule(dynamic, 16) reduction(+ : rows, checked, refused, bits_bad, code_bad, sub)
            for (int a = 1; a < 0x7f80; a += stride) {
                const float s = bf16((uint32_t)a) / full;
                const float r = 1.0f / s;
                rows++;
                for (uint32_t xb = 0; xb < 65536u; xb++) {
                    const float x = bf16(xb);
                    const bool nan = x != x;
                    if (!nan && !reng::fp8_product_ok(s, r, fabsf(x))) {
                        refused++;
                        continue;
                    }
                    if (nan && !reng::fp8_product_ok(s, r, 0.0f)) continue;
                    checked++;
                    const float q1 = reng::fp_quotient(x, s, r);
                    const float q0 = x / s;
                    const uint32_t b1 = reng::fp_bits(q1), b0 = reng::fp_bits(q0);
                    if ((b1 >> 31) != (reng::fp_bits(x) >> 31)) bits_bad++;
                    if (nan) {
                        if (q1 == q1) bits_bad++;
                    } else if (fabsf(x) >= 1.9721523e-31f && fabsf(q0) >= 1.17549435e-38f) {  // 2^-102, 2^-126
                        if (b1 != b0) bits_bad++;
                    } else {
                        sub++;  // codes only
                    }
                    if (b1 != b0) {  // equal bits encode equally: only differing pairs are encoded
                        for (int f = 0; f < 2; f++)
                            if (orc_fp8_encode(q1, f) != orc_fp8_encode(q0, f)) code_bad++;
                    }
                }
            }
        }
        printf("%s rows %lld checked %lld refused %lld subnormal %lld bits_mismatch %lld code_mismatch %lld\n",
               fmt == 0 ? "e4m3-scales" : "e5m2-scales", rows, checked, refused, sub, bits_bad, code_bad);
        bad_total += bits_bad + code_bad;
    }
    return bad_total ? 1 : 0;
}
