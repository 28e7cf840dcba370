/* Portable-C restatement of SLEEF 3.7 single-precision u10 exp / sin / cos.
 *
 * TEST INFRASTRUCTURE ONLY. This file belongs to the CPU oracle: it is linked
 * into the oracle restatement (liboracle) and into the reference build under
 * oracle/_ref (as the replacement for the NEON-only phonon_math.c). Product
 * code never links it.
 *
 * Published algorithm: N. Shibata and F. Petrogalli, "SLEEF: A Portable
 * Vectorized Library of C Standard Mathematical Functions", IEEE TPDS 31(6),
 * 2020; SLEEF 3.7.0 (BSL-1.0). The reference links the generated AdvSIMD
 * header (speech-mac vendor/sleef/sleefinline_advsimd.h): expf at :5589-5609,
 * sinf at :4926-4971, cosf at :4973-5020, the double-float helpers at
 * :4479-4590 and the Payne-Hanek style reduction rempif at :4748-4775.
 *
 * Lane semantics that matter for bit-exactness:
 *  - vmla/vfma are fused multiply-adds (vfmaq_f32), so they are fmaf() here;
 *    plain vector add/mul are unfused, so this file is built with
 *    -ffp-contract=off.
 *  - vrint is round-half-even (vrndnq_f32) == rintf() in the default mode.
 *  - sin/cos choose the cheap Cody-Waite reduction only when ALL FOUR lanes
 *    of the vector satisfy |d| < 125; otherwise every lane of the group takes
 *    the rempif path. oracle_sleef_sincosf4 keeps that group rule.
 *
 * Domain: the rempif path is restated for |d| < 2^25 only (one row of the
 * 2/pi table). RoPE phases are position*freq <= 8191 and the reference's own
 * pinned phases stay below 2^13, so the oracle never leaves that domain.
 * Inputs outside it return NaN so that a caller can never silently use them.
 */
#include "sleef_u10.h"

#include <math.h>
#include <stdint.h>
#include <string.h>

typedef struct {
    float x, y;
} df2;

static float bits_to_float(uint32_t b) {
    float f;
    memcpy(&f, &b, 4);
    return f;
}
static uint32_t float_to_bits(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    return b;
}
/* x with its sign flipped when y's sign bit is set (SLEEF vmulsign). */
static float mulsign(float x, float y) {
    return bits_to_float(float_to_bits(x) ^ (float_to_bits(y) & 0x80000000u));
}
static int32_t rint_to_int(float x) {
    return (int32_t)rintf(x);
}

/* ---- double-float arithmetic (SLEEF df* helpers) ---- */
static df2 df(float x, float y) {
    df2 r = {x, y};
    return r;
}
static df2 dfnormalize(df2 t) {
    float s = t.x + t.y;
    return df(s, (t.x - s) + t.y);
}
static df2 dfadd_f_f(float x, float y) {
    float s = x + y;
    return df(s, (x - s) + y);
}
static df2 dfadd2_f_f(float x, float y) {
    float s = x + y, v = s - x;
    return df(s, (x - (s - v)) + (y - v));
}
static df2 dfadd_df_f(df2 x, float y) {
    float s = x.x + y;
    return df(s, ((x.x - s) + y) + x.y);
}
static df2 dfadd2_df_f(df2 x, float y) {
    float s = x.x + y, v = s - x.x;
    float t = (x.x - (s - v)) + (y - v);
    return df(s, t + x.y);
}
static df2 dfadd_f_df(float x, df2 y) {
    float s = x + y.x;
    return df(s, ((x - s) + y.x) + y.y);
}
static df2 dfadd2_df_df(df2 x, df2 y) {
    float s = x.x + y.x, v = s - x.x;
    float t = (x.x - (s - v)) + (y.x - v);
    return df(s, t + (x.y + y.y));
}
static df2 dfmul_f_f(float x, float y) {
    float s = x * y;
    return df(s, fmaf(x, y, -s));
}
static df2 dfmul_df_f(df2 x, float y) {
    float s = x.x * y;
    return df(s, fmaf(x.y, y, fmaf(x.x, y, -s)));
}
static df2 dfmul_df_df(df2 x, df2 y) {
    float s = x.x * y.x;
    return df(s, fmaf(x.x, y.y, fmaf(x.y, y.x, fmaf(x.x, y.x, -s))));
}
static float dfmul_to_f(df2 x, df2 y) {
    return fmaf(x.x, y.x, fmaf(x.y, y.x, x.x * y.y));
}
static df2 dfsqu(df2 x) {
    float s = x.x * x.x;
    return df(s, fmaf(x.x + x.x, x.y, fmaf(x.x, x.x, -s)));
}

/* 2^q for q in the normal range, by building the exponent field. */
static float pow2i(int32_t q) {
    return bits_to_float((uint32_t)(q + 0x7f) << 23);
}

float oracle_sleef_expf(float d) {
    if (isnan(d))
        return d;
    int32_t q = rint_to_int(d * 1.442695040888963407359924681001892137f);
    float s = fmaf((float)q, -0.693145751953125f, d);
    s = fmaf((float)q, -1.428606765330187045e-06f, s);
    float u = 0.000198527617612853646278381f;
    u = fmaf(u, s, 0.00139304355252534151077271f);
    u = fmaf(u, s, 0.00833336077630519866943359f);
    u = fmaf(u, s, 0.0416664853692054748535156f);
    u = fmaf(u, s, 0.166666671633720397949219f);
    u = fmaf(u, s, 0.5f);
    u = 1.0f + fmaf(s * s, u, s);
    /* vldexp2: split the exponent so each factor stays representable. */
    int32_t half = q >> 1;
    u = (u * pow2i(half)) * pow2i(q - half);
    if (d < -104.0f)
        u = 0.0f;
    if (100.0f < d)
        u = INFINITY;
    return u;
}

/* Reduction argument result: r = d mod pi/2 as a double-float, and the
 * quadrant information i (SLEEF dfi_t). */
typedef struct {
    df2 r;
    int32_t i;
} dfi;

/* rempisubf: split x into (x - round(4x)/4, quadrant steps). */
static float rempisub(float x, int32_t *steps) {
    float y = rintf(x * 4.0f);
    *steps = (int32_t)truncf(y - rintf(x) * 4.0f);
    return x - y * 0.25f;
}

/* First row (exponent bucket 0) of SLEEF's float Payne-Hanek table: four
 * floats whose sum is 1/(2*pi) to within 6e-30, each with trailing zero bits
 * so that products with the argument are exact enough. Valid for |a| < 2^25. */
static const float inv_2pi_pieces[4] = {0.159154892f, 5.112411827e-08f, 3.626141271e-15f,
                                        -2.036222915e-22f};

static dfi rempif(float a) {
    df2 x, y;
    int32_t q, steps;
    x = dfmul_f_f(a, inv_2pi_pieces[0]);
    x.x = rempisub(x.x, &steps);
    q = steps;
    x = dfnormalize(x);
    y = dfmul_f_f(a, inv_2pi_pieces[1]);
    x = dfadd2_df_df(x, y);
    x.x = rempisub(x.x, &steps);
    q += steps;
    x = dfnormalize(x);
    y = dfmul_df_f(df(inv_2pi_pieces[2], inv_2pi_pieces[3]), a);
    x = dfadd2_df_df(x, y);
    x = dfnormalize(x);
    x = dfmul_df_df(x, df(3.1415927410125732422f * 2, -8.7422776573475857731e-08f * 2));
    if (fabsf(a) < 0.7f)
        x = df(a, 0.0f);
    dfi r = {x, q};
    return r;
}

/* Shared tail of sin and cos: t * (1 + s*(-1/6 + s*poly(s))) evaluated in
 * double-float, with s = t^2. */
static float sincos_kernel(df2 s_in) {
    df2 t = s_in, s = dfsqu(s_in);
    float u = 2.6083159809786593541503e-06f;
    u = fmaf(u, s.x, -0.0001981069071916863322258f);
    u = fmaf(u, s.x, 0.00833307858556509017944336f);
    df2 x = dfadd_f_df(1.0f, dfmul_df_df(dfadd_f_f(-0.166666597127914428710938f, u * s.x), s));
    return dfmul_to_f(t, x);
}

static const float kRempifLimit = 33554432.0f; /* 2^25 */

static float sinf_lane(float d, int fast) {
    int32_t q;
    df2 s;
    if (fast) {
        float u = rintf(d * 0.318309886183790671537767526745028724f);
        q = rint_to_int(u);
        float v = fmaf(u, -3.1414794921875f, d);
        s = dfadd2_f_f(v, u * -0.00011315941810607910156f);
        s = dfadd_df_f(s, u * -1.9841872589410058936e-09f);
    } else {
        if (!(fabsf(d) < kRempifLimit))
            return NAN;
        dfi r = rempif(d);
        q = r.i & 3;
        q = q + q + (r.r.x > 0 ? 2 : 1);
        q >>= 2;
        if ((r.i & 1) == 1) {
            df2 x = df(mulsign(3.1415927410125732422f * -0.5f, r.r.x),
                       mulsign(-8.7422776573475857731e-08f * -0.5f, r.r.x));
            r.r = dfadd2_df_df(r.r, x);
        }
        s = dfnormalize(r.r);
    }
    float u = sincos_kernel(s);
    if ((q & 1) == 1)
        u = -u;
    if (float_to_bits(d) == 0x80000000u)
        u = d;
    return u;
}

static float cosf_lane(float d, int fast) {
    int32_t q;
    df2 s;
    if (fast) {
        float dq =
            fmaf(rintf(fmaf(d, 0.318309886183790671537767526745028724f, -0.5f)), 2.0f, 1.0f);
        q = rint_to_int(dq);
        s = dfadd2_f_f(d, dq * (-3.1414794921875f * 0.5f));
        s = dfadd2_df_f(s, dq * (-0.00011315941810607910156f * 0.5f));
        s = dfadd2_df_f(s, dq * (-1.9841872589410058936e-09f * 0.5f));
    } else {
        if (!(fabsf(d) < kRempifLimit))
            return NAN;
        dfi r = rempif(d);
        q = r.i & 3;
        q = q + q + (r.r.x > 0 ? 8 : 7);
        q >>= 1;
        if ((r.i & 1) == 0) {
            float y = r.r.x > 0 ? 0.0f : -1.0f;
            df2 x = df(mulsign(3.1415927410125732422f * -0.5f, y),
                       mulsign(-8.7422776573475857731e-08f * -0.5f, y));
            r.r = dfadd2_df_df(r.r, x);
        }
        s = dfnormalize(r.r);
    }
    float u = sincos_kernel(s);
    if ((q & 2) == 0)
        u = -u;
    return u;
}

void oracle_sleef_sincosf4(const float d[4], float cosines[4], float sines[4]) {
    int fast = 1;
    for (int lane = 0; lane < 4; lane++)
        if (!(fabsf(d[lane]) < 125.0f))
            fast = 0;
    for (int lane = 0; lane < 4; lane++) {
        if (isnan(d[lane]) || isinf(d[lane])) {
            cosines[lane] = sines[lane] = NAN;
            continue;
        }
        sines[lane] = sinf_lane(d[lane], fast);
        cosines[lane] = cosf_lane(d[lane], fast);
    }
}

void oracle_sleef_expf4(float values[4]) {
    for (int lane = 0; lane < 4; lane++)
        values[lane] = oracle_sleef_expf(values[lane]);
}
