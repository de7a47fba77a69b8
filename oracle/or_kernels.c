/*
 * Oracle kernels — TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * Each function restates a reference kernel with its float32 operation order. The "avx2" forms
 * follow the Go-assembler kernels of internal/kernels/vec_amd64.s instruction by instruction
 * (fused multiply-adds where the assembly uses VFMADD/VFNMADD, separate multiply and add in its
 * scalar tails); the "pure" forms follow the pure-Go fallbacks of internal/kernels/int8.go and
 * vec_ops.go. Build with -ffp-contract=off so that the compiler adds no fusion of its own.
 */
#include "oracle.h"

#include <math.h>
#include <string.h>
#if defined(__AVX2__) && defined(__FMA__)
#include <immintrin.h>
#define OR_HAVE_AVX2 1
#else
#define OR_HAVE_AVX2 0
#endif

static int g_avx2 = OR_HAVE_AVX2;

void or_set_avx2(int on) { g_avx2 = on && OR_HAVE_AVX2; }
int or_get_avx2(void) { return g_avx2; }

/* Horizontal sum of the 8 lanes a0..a7 as vec_amd64.s does it (VEXTRACTF128, VADDPS,
 * VSHUFPS $0x4E, VADDPS, VSHUFPS $0x01, VADDSS): ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)). */
static float hsum8(const float a[8]) {
    float b0 = a[0] + a[4], b1 = a[1] + a[5], b2 = a[2] + a[6], b3 = a[3] + a[7];
    float c0 = b0 + b2, c1 = b1 + b3;
    return c0 + c1;
}

/* ---- DotInt8F32: int8.go:8-29, vec_amd64.s:603-679 ---- */
static float dot_i8_pure(const float* x, const int8_t* w, int n) {
    float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    int j = 0;
    for (; j <= n - 4; j += 4) {
        s0 += x[j] * (float)w[j];
        s1 += x[j + 1] * (float)w[j + 1];
        s2 += x[j + 2] * (float)w[j + 2];
        s3 += x[j + 3] * (float)w[j + 3];
    }
    for (; j < n; j++) s0 += x[j] * (float)w[j];
    return (s0 + s1) + (s2 + s3);
}

static float dot_i8_avx2_order(const float* x, const int8_t* w, int n) {
    /* Scalar statement of the assembly: 4 accumulators of 8 lanes over 32-blocks, further
     * 8-blocks into the first, the reduction above, then a scalar tail (VMULSS + VADDSS). */
    float y0[8] = {0}, y1[8] = {0}, y4[8] = {0}, y5[8] = {0};
    int i = 0;
    for (; n - i >= 32; i += 32) {
        for (int l = 0; l < 8; l++) {
            y0[l] = fmaf((float)w[i + l], x[i + l], y0[l]);
            y1[l] = fmaf((float)w[i + 8 + l], x[i + 8 + l], y1[l]);
            y4[l] = fmaf((float)w[i + 16 + l], x[i + 16 + l], y4[l]);
            y5[l] = fmaf((float)w[i + 24 + l], x[i + 24 + l], y5[l]);
        }
    }
    for (; n - i >= 8; i += 8)
        for (int l = 0; l < 8; l++) y0[l] = fmaf((float)w[i + l], x[i + l], y0[l]);
    float a[8];
    for (int l = 0; l < 8; l++) a[l] = (y0[l] + y1[l]) + (y4[l] + y5[l]);
    float s = hsum8(a);
    for (; i < n; i++) {
        float t = (float)w[i] * x[i];
        s = s + t;
    }
    return s;
}

#if OR_HAVE_AVX2
static float hsum8_v(__m256 v) {
    float a[8];
    _mm256_storeu_ps(a, v);
    return hsum8(a);
}

static float dot_i8_avx2(const float* x, const int8_t* w, int n) {
    __m256 y0 = _mm256_setzero_ps(), y1 = y0, y4 = y0, y5 = y0;
    int i = 0;
    for (; n - i >= 32; i += 32) {
        __m256 w0 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i*)(w + i))));
        __m256 w1 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i*)(w + i + 8))));
        __m256 w2 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i*)(w + i + 16))));
        __m256 w3 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i*)(w + i + 24))));
        y0 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(x + i), y0);
        y1 = _mm256_fmadd_ps(w1, _mm256_loadu_ps(x + i + 8), y1);
        y4 = _mm256_fmadd_ps(w2, _mm256_loadu_ps(x + i + 16), y4);
        y5 = _mm256_fmadd_ps(w3, _mm256_loadu_ps(x + i + 24), y5);
    }
    for (; n - i >= 8; i += 8) {
        __m256 w0 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i*)(w + i))));
        y0 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(x + i), y0);
    }
    y0 = _mm256_add_ps(y0, y1);
    y4 = _mm256_add_ps(y4, y5);
    y0 = _mm256_add_ps(y0, y4);
    float s = hsum8_v(y0);
    for (; i < n; i++) {
        float t = (float)w[i] * x[i];
        s = s + t;
    }
    return s;
}
#endif

float or_dot_i8_f32(const float* x, const int8_t* w, int n) {
    if (n <= 0) return 0.0f;
    if (!g_avx2) return dot_i8_pure(x, w, n);
#if OR_HAVE_AVX2
    return dot_i8_avx2(x, w, n);
#else
    return dot_i8_avx2_order(x, w, n);
#endif
}

/* Exposed for the equivalence test of the intrinsic and scalar statements of the assembly. */
float or_dot_i8_f32_scalar_order(const float* x, const int8_t* w, int n) { return dot_i8_avx2_order(x, w, n); }

/* ---- DotF32: vec_ops.go:35-60, vec_amd64.s:4-64 ---- */
static float dot_f32_pure(const float* x, const float* y, int n) {
    float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    int j = 0;
    for (; j <= n - 4; j += 4) {
        s0 += x[j] * y[j];
        s1 += x[j + 1] * y[j + 1];
        s2 += x[j + 2] * y[j + 2];
        s3 += x[j + 3] * y[j + 3];
    }
    for (; j < n; j++) s0 += x[j] * y[j];
    return (s0 + s1) + (s2 + s3);
}

static float dot_f32_avx2_order(const float* x, const float* y, int n) {
    float a0[8] = {0}, a1[8] = {0};
    int i = 0;
    for (; n - i >= 16; i += 16)
        for (int l = 0; l < 8; l++) {
            a0[l] = fmaf(x[i + l], y[i + l], a0[l]);
            a1[l] = fmaf(x[i + 8 + l], y[i + 8 + l], a1[l]);
        }
    if (n - i >= 8) {
        for (int l = 0; l < 8; l++) a0[l] = fmaf(x[i + l], y[i + l], a0[l]);
        i += 8;
    }
    float a[8];
    for (int l = 0; l < 8; l++) a[l] = a0[l] + a1[l];
    float s = hsum8(a);
    for (; i < n; i++) {
        float t = x[i] * y[i];
        s = s + t;
    }
    return s;
}

float or_dot_f32(const float* x, const float* y, int n) {
    if (n <= 0) return 0.0f;
    if (!g_avx2) return dot_f32_pure(x, y, n);
#if OR_HAVE_AVX2
    __m256 a0 = _mm256_setzero_ps(), a1 = a0;
    int i = 0;
    for (; n - i >= 16; i += 16) {
        a0 = _mm256_fmadd_ps(_mm256_loadu_ps(x + i), _mm256_loadu_ps(y + i), a0);
        a1 = _mm256_fmadd_ps(_mm256_loadu_ps(x + i + 8), _mm256_loadu_ps(y + i + 8), a1);
    }
    if (n - i >= 8) {
        a0 = _mm256_fmadd_ps(_mm256_loadu_ps(x + i), _mm256_loadu_ps(y + i), a0);
        i += 8;
    }
    float s = hsum8_v(_mm256_add_ps(a0, a1));
    for (; i < n; i++) {
        float t = x[i] * y[i];
        s = s + t;
    }
    return s;
#else
    return dot_f32_avx2_order(x, y, n);
#endif
}

float or_dot_f32_scalar_order(const float* x, const float* y, int n) { return dot_f32_avx2_order(x, y, n); }

/* ---- AddScaledF32: vec_ops.go:62-88, vec_amd64.s:66-123 ---- */
void or_add_scaled_f32(float* y, const float* x, float alpha, int n) {
    if (n <= 0) return;
    int j = 0;
    if (!g_avx2) {
        for (; j <= n - 4; j += 4) {
            y[j] += alpha * x[j];
            y[j + 1] += alpha * x[j + 1];
            y[j + 2] += alpha * x[j + 2];
            y[j + 3] += alpha * x[j + 3];
        }
        for (; j < n; j++) y[j] += alpha * x[j];
        return;
    }
    for (; n - j >= 16; j += 16)
        for (int l = 0; l < 16; l++) y[j + l] = fmaf(alpha, x[j + l], y[j + l]);
    if (n - j >= 8) {
        for (int l = 0; l < 8; l++) y[j + l] = fmaf(alpha, x[j + l], y[j + l]);
        j += 8;
    }
    for (; j < n; j++) {
        float t = x[j] * alpha;
        y[j] = t + y[j];
    }
}

/* ---- FastExpF32 (vec_ops.go:104-138) and the vectorised exp of vec_amd64.s:282-431 ---- */
static float bits_f32(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

float or_fast_exp_f32(float x) {
    /* Pure-Go FastExpF32: no fusion, k rounded half away from zero (math.Round). */
    if (x < -88.0f) return 0.0f;
    if (x > 88.0f) return 3.4028235e+38f;
    const float invLn2 = (float)1.4426950408889634;
    const float ln2Hi = 0.693145751953125f;
    const float ln2Lo = (float)1.4286068203094172e-06;
    float k = (float)round((double)(x * invLn2));
    if (k > 127) k = 127;
    else if (k < -126) k = -126;
    float r = x - k * ln2Hi - k * ln2Lo;
    const float c2 = 0.5f, c3 = 0.16666667f, c4 = 0.041666668f, c5 = 0.008333334f;
    float poly = 1.0f + r * (1.0f + r * (c2 + r * (c3 + r * (c4 + r * c5))));
    int ki = (int)k + 127;
    if (ki <= 0) return 0.0f;
    if (ki >= 255) return 3.4028235e+38f;
    return poly * bits_f32((uint32_t)ki << 23);
}

/* One lane of vecExpASM_F32: clamp to [-88, 88] (VMINPS/VMAXPS), k = round-to-nearest-even of
 * x*invLn2 (VROUNDPS $0), r by two fused negated multiply-adds, the degree-5 polynomial by fused
 * Horner steps, and 2^k built from the exponent bits. */
static float exp_asm_lane(float x) {
    const float c88 = bits_f32(0x42b00000u), cm88 = bits_f32(0xc2b00000u);
    const float invLn2 = bits_f32(0x3fb8aa3bu), ln2Hi = bits_f32(0x3f317200u), ln2Lo = bits_f32(0x35bfbe8eu);
    const float c5 = bits_f32(0x3c088889u), c4 = bits_f32(0x3d2aaaabu), c3 = bits_f32(0x3e2aaaabu);
    const float c2 = bits_f32(0x3f000000u), one = 1.0f;
    x = x < c88 ? x : c88;   /* VMINPS: min(x, 88) */
    x = x > cm88 ? x : cm88; /* VMAXPS: max(x, -88) */
    float k = nearbyintf(x * invLn2);
    float r = fmaf(-k, ln2Hi, x);
    r = fmaf(-k, ln2Lo, r);
    float p = fmaf(c5, r, c4);
    p = fmaf(p, r, c3);
    p = fmaf(p, r, c2);
    p = fmaf(p, r, one);
    p = fmaf(p, r, one);
    int32_t ki = (int32_t)k + 127;
    uint32_t bits = (uint32_t)ki << 23;
    return p * bits_f32(bits);
}

void or_vec_exp_f32(float* dst, const float* src, int n) {
    if (!g_avx2) {
        for (int i = 0; i < n; i++) dst[i] = or_fast_exp_f32(src[i]);
        return;
    }
    for (int i = 0; i < n; i++) dst[i] = exp_asm_lane(src[i]);
}

/* ---- MatVecInt8 (int8.go:31-41) ---- */
void or_matvec_i8(float* y, int rows, const int8_t* w, int stride, float scale, const float* x, int cols,
                  const float* bias) {
    for (int r = 0; r < rows; r++) {
        float v = or_dot_i8_f32(x, w + (size_t)r * stride, cols) * scale;
        if (bias) v += bias[r];
        y[r] = v;
    }
}

/* ---- RMSNormForwardF32 (nn/rmsnorm.go:14-32) ---- */
float or_rmsnorm_f32(const float* x, const float* gamma, float* out, float* xhat, int d, float eps) {
    if (d == 0) return 1.0f;
    float sumsq = or_dot_f32(x, x, d);
    float ms = sumsq / (float)d;
    ms = ms + eps;
    float rms = (float)sqrt((double)ms);
    float inv = 1.0f / rms;
    for (int i = 0; i < d; i++) {
        float hat = x[i] * inv;
        if (xhat) xhat[i] = hat;
        out[i] = hat * gamma[i];
    }
    return rms;
}

/* ---- SoftmaxInPlaceF32 (nn/head.go:93-111) ---- */
void or_softmax_f32(float* logits, float* scratch, int n) {
    float mx = -3.40282346638528859811704183484516925440e+38f;
    for (int i = 0; i < n; i++)
        if (logits[i] > mx) mx = logits[i];
    for (int i = 0; i < n; i++) scratch[i] = logits[i] - mx;
    or_vec_exp_f32(logits, scratch, n);
    float sum = 0.0f;
    for (int i = 0; i < n; i++) sum += logits[i];
    float inv = 1.0f / sum;
    for (int i = 0; i < n; i++) logits[i] *= inv;
}

/* ---- sigmoidClamped (quant/stream.go:128-136) ---- */
float or_sigmoid_clamped(float x) {
    if (x > 15.0f) return 1.0f;
    if (x < -15.0f) return 0.0f;
    float e = (float)exp((double)(-x));
    return 1.0f / (1.0f + e);
}

/* ---- ca helpers ---- */
int or_step_dilation(int initial, int base, int step) {
    int d = initial;
    for (int s = 0; s < step && d < 32; s++) d *= base;
    return d < 32 ? d : 32;
}

/* ComputeSelectiveLatchBaseLogits (ca/latch.go:11-25) over ComputeDecayLatchConstants
 * (ca/layout.go:63-85): half-lives geometric from 1.5 to 64 tokens, lambda = 2^(-1/T),
 * base = log(lambda / (1 - lambda)) with lambda widened from float32. */
void or_latch_base_logits(int d, float* out) {
    const double minT = 1.5, maxT = 64.0;
    for (int i = 0; i < d; i++) {
        double td;
        if (d == 1) td = minT;
        else {
            double ratio = pow(maxT / minT, 1.0 / (double)(d - 1));
            td = minT * pow(ratio, (double)i);
        }
        float lam32 = (float)pow(2.0, -1.0 / td);
        double lam = (double)lam32;
        if (lam <= 0.0) out[i] = -15.0f;
        else if (lam >= 1.0) out[i] = 15.0f;
        else out[i] = (float)log(lam / (1.0 - lam));
    }
}

/* ---- NewTensorF32 (quant/tensor.go:12-42): returns the scale ---- */
float or_quantize_tensor(const float* w, size_t n, int8_t* out) {
    if (n == 0) return 0.0f;
    float maxabs = 0.0f;
    for (size_t i = 0; i < n; i++) {
        float a = (float)fabs((double)w[i]);
        if (a > maxabs) maxabs = a;
    }
    if (maxabs == 0.0f) {
        memset(out, 0, n);
        return 1.0f;
    }
    float scale = maxabs / 127.0f;
    for (size_t i = 0; i < n; i++) {
        float q = w[i] / scale;
        double v = round((double)q);
        if (v > 127) v = 127;
        else if (v < -127) v = -127;
        out[i] = (int8_t)v;
    }
    return scale;
}
