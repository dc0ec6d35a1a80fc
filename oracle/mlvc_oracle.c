/*
 * CPU restatement of the reference FP16 conv-stack arithmetic (test
 * infrastructure only; see mlvc_oracle.h for the citations).  Compiled with
 * -ffp-contract=off so every multiply and add rounds to FP32 separately.
 */
#include "mlvc_oracle.h"

#include <math.h>
#include <string.h>

static uint32_t f2u(float f)
{
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

static float u2f(uint32_t u)
{
    float f;
    memcpy(&f, &u, 4);
    return f;
}

float oracle_half_to_float(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1fu;
    const uint32_t man = h & 0x3ffu;
    if (exp == 0) {
        /* zero or subnormal: value = man * 2^-24, exact in FP32 */
        const float mag = (float)man * u2f(0x33800000u); /* 2^-24 */
        return sign ? -mag : mag;
    }
    if (exp == 31)
        return u2f(sign | 0x7f800000u | (man << 13) | (man ? 0x00400000u : 0u));
    return u2f(sign | ((exp + 112u) << 23) | (man << 13));
}

uint16_t oracle_float_to_half(float f)
{
    const uint32_t u = f2u(f);
    const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    const uint32_t exp = (u >> 23) & 0xffu;
    uint32_t man = u & 0x7fffffu;
    if (exp == 0xff)
        return (uint16_t)(sign | 0x7c00u | (man ? (0x200u | (man >> 13)) : 0u));
    int e = (int)exp - 127 + 15;
    if (e >= 31)
        return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10)
            return sign; /* below half the smallest subnormal: rounds to zero */
        man |= 0x800000u;
        const unsigned shift = (unsigned)(14 - e);
        uint32_t q = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u)))
            ++q;
        return (uint16_t)(sign | q); /* carry into the exponent is correct */
    }
    uint32_t q = man >> 13;
    const uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) {
        ++q;
        if (q == 0x400u) {
            q = 0;
            ++e;
            if (e >= 31)
                return (uint16_t)(sign | 0x7c00u);
        }
    }
    return (uint16_t)(sign | ((uint32_t)e << 10) | q);
}

void oracle_halves_to_floats(const uint16_t* src, float* dst, size_t n)
{
    for (size_t i = 0; i < n; ++i)
        dst[i] = oracle_half_to_float(src[i]);
}

void oracle_floats_to_halves(const float* src, uint16_t* dst, size_t n)
{
    for (size_t i = 0; i < n; ++i)
        dst[i] = oracle_float_to_half(src[i]);
}

static float rh(float v) { return oracle_half_to_float(oracle_float_to_half(v)); }

void oracle_conv2d(const uint16_t* x, const uint16_t* w, const uint16_t* bias,
                   uint16_t* y, int n, int ic, int ih, int iw, int oc, int oh,
                   int ow, int kh, int kw, int sh, int sw, int ph, int pw,
                   int groups, int epilogue, float alpha,
                   const uint16_t* residual)
{
    const int icg = ic / groups;
    const int ocg = oc / groups;
    for (int b = 0; b < n; ++b)
        for (int o = 0; o < oc; ++o) {
            const int g = o / ocg;
            const float b0 = bias ? oracle_half_to_float(bias[o]) : 0.0f;
            for (int yy = 0; yy < oh; ++yy)
                for (int xx = 0; xx < ow; ++xx) {
                    float acc = b0;
                    for (int ky = 0; ky < kh; ++ky) {
                        const int sy = yy * sh + ky - ph;
                        if (sy < 0 || sy >= ih)
                            continue;
                        for (int kx = 0; kx < kw; ++kx) {
                            const int sx = xx * sw + kx - pw;
                            if (sx < 0 || sx >= iw)
                                continue;
                            for (int c = 0; c < icg; ++c) {
                                const float xv = oracle_half_to_float(
                                    x[(((size_t)b * ic + g * icg + c) * ih + sy) * iw + sx]);
                                const float wv = oracle_half_to_float(
                                    w[(((size_t)o * icg + c) * kh + ky) * kw + kx]);
                                const float p = xv * wv;
                                acc = acc + p;
                            }
                        }
                    }
                    const size_t oi = (((size_t)b * oc + o) * oh + yy) * ow + xx;
                    float v = rh(acc);
                    if (epilogue == 1 && v < 0.0f)
                        v = rh(v * alpha);
                    else if (epilogue == 2)
                        v = rh(v + oracle_half_to_float(residual[oi]));
                    y[oi] = oracle_float_to_half(v);
                }
        }
}

void oracle_unary(const uint16_t* x, uint16_t* y, size_t count, int op,
                  float alpha, float lo, float hi)
{
    for (size_t i = 0; i < count; ++i) {
        const float v = oracle_half_to_float(x[i]);
        float r = v;
        switch (op) {
        case 0: r = v >= 0.0f ? v : alpha * v; break;
        case 1: r = fminf(fmaxf(v, lo), hi); break;
        case 2: r = 1.0f / (1.0f + expf(-v)); break;
        case 3: r = 1.0f / v; break;
        case 4: r = nearbyintf(v); break;
        default: break;
        }
        y[i] = oracle_float_to_half(r);
    }
}

void oracle_binary(const uint16_t* a, const uint16_t* b, uint16_t* y,
                   const int64_t* od, const int64_t* ad, const int64_t* bd,
                   int op)
{
    int64_t as[4], bs[4];
    as[3] = ad[3] == 1 ? 0 : 1;
    as[2] = ad[2] == 1 ? 0 : ad[3];
    as[1] = ad[1] == 1 ? 0 : ad[2] * ad[3];
    as[0] = ad[0] == 1 ? 0 : ad[1] * ad[2] * ad[3];
    bs[3] = bd[3] == 1 ? 0 : 1;
    bs[2] = bd[2] == 1 ? 0 : bd[3];
    bs[1] = bd[1] == 1 ? 0 : bd[2] * bd[3];
    bs[0] = bd[0] == 1 ? 0 : bd[1] * bd[2] * bd[3];
    size_t i = 0;
    for (int64_t c0 = 0; c0 < od[0]; ++c0)
        for (int64_t c1 = 0; c1 < od[1]; ++c1)
            for (int64_t c2 = 0; c2 < od[2]; ++c2)
                for (int64_t c3 = 0; c3 < od[3]; ++c3, ++i) {
                    const float va = oracle_half_to_float(
                        a[c0 * as[0] + c1 * as[1] + c2 * as[2] + c3 * as[3]]);
                    const float vb = oracle_half_to_float(
                        b[c0 * bs[0] + c1 * bs[1] + c2 * bs[2] + c3 * bs[3]]);
                    const float r = op == 0 ? va + vb : op == 1 ? va * vb : va - vb;
                    y[i] = oracle_float_to_half(r);
                }
}
