/*
 * CPU oracle for the fake-quantization path -- TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, element by element, the reference's own PyTorch CPU implementation
 * of QATFactory's quantizers (qatfactory/quant/formats/{nvfp4,mxfp4,q4_k}.py) as plain C,
 * so that the CUDA kernels in qatfactory_b200/csrc can be checked bit for bit.  Only the
 * tests, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it; the product
 * path never does.  It is pinned against golden vectors generated from the reference
 * itself (tests/golden/make_golden.py) and against the reference tests' known answers.
 *
 * Floating-point rules: every operation below is one IEEE binary32 operation in the order
 * the reference's torch expression evaluates it (compile with -ffp-contract=off, no
 * -ffast-math; x86-64 evaluates float in SSE registers, FLT_EVAL_METHOD == 0).  Torch
 * idioms that are not what they look like are spelled out where they occur:
 *   - `c / tensor` is `tensor.reciprocal() * c` (torch/_tensor.py __rdiv__), i.e. two
 *     roundings, not one true division;
 *   - `tensor.sign()` is +0 for -0 and for NaN;
 *   - a float32 row sum over 32 contiguous elements on the reference host adds 8-lane
 *     vectors: t[k] = ((x[k] + x[k+8]) + x[k+16]) + x[k+24], then 0 + t[0] + ... + t[7]
 *     sequentially (probed against torch 2.11 on the build host; see make_golden.py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2 };

/* ---------------------------------------------------------------- scalar conversions */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

static float half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t exp = (h >> 10) & 0x1F;
    uint32_t man = h & 0x3FF;
    if (exp == 0) {
        if (man == 0) return u2f(sign);
        /* subnormal: value = man * 2^-24, exact in float */
        float v = (float)man * 5.9604644775390625e-08f;
        return sign ? -v : v;
    }
    if (exp == 31) return u2f(sign | 0x7F800000u | (man << 13));
    return u2f(sign | ((exp + 112) << 23) | (man << 13));
}

/* float -> IEEE half, round to nearest even, overflow to inf (torch c10::Half semantics). */
static uint16_t float_to_half(float f) {
    uint32_t x = f2u(f);
    uint32_t sign = (x >> 16) & 0x8000;
    uint32_t ax = x & 0x7FFFFFFF;
    if (ax > 0x7F800000) return (uint16_t)(sign | 0x7E00); /* NaN */
    if (ax >= 0x477FF000) return (uint16_t)(sign | 0x7C00); /* >= 65520 rounds to inf */
    if (ax < 0x38800000) {
        /* result is a half subnormal (or zero): units of 2^-24 */
        float a = u2f(ax);
        float scaled = a * 16777216.0f; /* exact: multiply by 2^24 */
        float r = nearbyintf(scaled);   /* ties to even in the default mode */
        return (uint16_t)(sign | (uint32_t)r);
    }
    /* normal: drop 13 mantissa bits with ties-to-even */
    uint32_t rounded = ax + 0xFFF + ((ax >> 13) & 1);
    return (uint16_t)(sign | ((rounded - 0x38000000u) >> 13));
}

static inline float bf16_to_float(uint16_t b) { return u2f((uint32_t)b << 16); }

/* float -> bfloat16, round to nearest even (c10::BFloat16 round_to_nearest_even). */
static inline uint16_t float_to_bf16(float f) {
    if (isnan(f)) return 0x7FC0;
    uint32_t u = f2u(f);
    u += 0x7FFF + ((u >> 16) & 1);
    return (uint16_t)(u >> 16);
}

static inline float load_elem(const void *p, int dtype, int64_t i) {
    switch (dtype) {
    case DT_F32: return ((const float *)p)[i];
    case DT_F16: return half_to_float(((const uint16_t *)p)[i]);
    default: return bf16_to_float(((const uint16_t *)p)[i]);
    }
}

static inline void store_elem(void *p, int dtype, int64_t i, float v) {
    switch (dtype) {
    case DT_F32: ((float *)p)[i] = v; break;
    case DT_F16: ((uint16_t *)p)[i] = float_to_half(v); break;
    default: ((uint16_t *)p)[i] = float_to_bf16(v); break;
    }
}

/* Running max / min of torch's CPU reductions: NaN propagates and, between equal values
 * (+0 and -0), the earlier one is kept (probed: max over [-0., +0.] is -0.). `acc` is the
 * running value, `x` the next element. */
static inline float nanmax(float acc, float x) {
    if (isnan(acc) || isnan(x)) return NAN;
    return x > acc ? x : acc;
}

static inline float nanmin(float acc, float x) {
    if (isnan(acc) || isnan(x)) return NAN;
    return x < acc ? x : acc;
}

/* torch.clamp(v, max=0) and torch.minimum(v, 0): a zero or NaN v is kept as it is. */
static inline float clamp_max0(float v) { return v > 0.0f ? 0.0f : v; }

/* torch.clamp(v, lo, hi): NaN passes through */
static inline float clampf(float v, float lo, float hi) {
    if (isnan(v)) return v;
    return v < lo ? lo : (v > hi ? hi : v);
}

/* ------------------------------------------------------------------- E2M1 and E4M3 */

static const float E2M1_LEVELS[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
static const float E2M1_BOUNDS[7] = {0.25f, 0.75f, 1.25f, 1.75f, 2.5f, 3.5f, 5.0f};

/* _round_to_e2m1 (nvfp4.py:44-52): bucketize(|v|, bounds, right=False), exact ties move an
 * odd index up by one, then codebook[index] * sign(v).  Returns the magnitude index via
 * *index_out (0..7) so the packers can reuse it. */
static float round_to_e2m1(float v, int *index_out) {
    float m = fabsf(v);
    int idx;
    if (isnan(m)) {
        idx = 7; /* torch.bucketize places NaN past the last boundary */
    } else {
        idx = 0;
        while (idx < 7 && E2M1_BOUNDS[idx] < m) idx++;
        int b = idx < 6 ? idx : 6;
        int tie = (idx < 7) && (m == E2M1_BOUNDS[b]);
        if (tie && (idx & 1)) idx++;
    }
    if (index_out) *index_out = idx;
    float sgn = (v > 0.0f) ? 1.0f : ((v < 0.0f) ? -1.0f : 0.0f); /* torch.sign: 0 for +-0, NaN */
    return E2M1_LEVELS[idx] * sgn;
}

/* _e2m1_values_to_indices (nvfp4.py:67-73): sign<<3 | level index; -0 encodes as 0. */
static inline uint8_t e2m1_nibble(float code_value, int level_index) {
    int negative = (code_value < 0.0f) && (level_index != 0);
    return (uint8_t)((negative << 3) | level_index);
}

/* float -> float8_e4m3fn -> float after clamp to [0, 448] (nvfp4.py:55-64), RNE with
 * subnormals (smallest 2^-9).  Returns the stored byte through *byte_out. */
static float cast_e4m3(float v, uint8_t *byte_out) {
    if (isnan(v)) { if (byte_out) *byte_out = 0x7F; return v; }
    v = clampf(v, 0.0f, 448.0f);
    uint32_t bits = f2u(v);
    int exp = (int)((bits >> 23) & 0xFF) - 127;
    if (v < 0.015625f) { /* below 2^-6: units of 2^-9 */
        float units = nearbyintf(v * 512.0f);
        if (byte_out) *byte_out = (uint8_t)units; /* 0..8; 8 is also the encoding of 2^-6 */
        return units * 0.001953125f;
    }
    uint32_t rounded = (bits + 0x7FFFF + ((bits >> 20) & 1)) & 0xFFF00000u;
    float r = u2f(rounded);
    exp = (int)((rounded >> 23) & 0xFF) - 127;
    if (byte_out) *byte_out = (uint8_t)(((exp + 7) << 3) | ((rounded >> 20) & 7));
    return r;
}

/* ----------------------------------------------------------------------------- amax */

/* weight.detach().abs().amax().float() (nvfp4.py:531) */
float oracle_tensor_amax(const void *x, int dtype, int64_t n) {
    float m = 0.0f;
    for (int64_t i = 0; i < n; i++) m = nanmax(m, fabsf(load_elem(x, dtype, i)));
    return m;
}

/* ---------------------------------------------------------------------------- NVFP4 */

#define NV_BLOCK 16

/* Block scales of one NVFP4 block (nvfp4.py:483-491 / :437-445).  Writes the dequant scale
 * (block_scale * global_scale) and the stored E4M3 byte. */
static float nvfp4_block_scale(float block_amax, float global_scale, uint8_t *scale_byte) {
    float denom = global_scale * 6.0f;
    float q = block_amax / denom;
    float bs = cast_e4m3(q, scale_byte);
    if (bs == 0.0f) { bs = 0.001953125f; if (scale_byte) *scale_byte = 0x01; }
    return bs * global_scale;
}

/* _fake_quantize_nvfp4_torch (nvfp4.py:465-501): y has the input dtype, mask one byte per
 * element (0/1).  Rows are padded with zeros to a multiple of 16 (nvfp4.py:475-477). */
void oracle_nvfp4_qdq(const void *x, int dtype, int64_t rows, int64_t cols, float tensor_amax,
                      void *y, uint8_t *mask) {
    if (tensor_amax == 0.0f) { /* nvfp4.py:493-494 */
        for (int64_t i = 0; i < rows * cols; i++) { store_elem(y, dtype, i, 0.0f); if (mask) mask[i] = 1; }
        return;
    }
    float gs = tensor_amax / 2688.0f;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        for (int64_t c0 = 0; c0 < cols; c0 += NV_BLOCK) {
            int64_t c1 = c0 + NV_BLOCK < cols ? c0 + NV_BLOCK : cols;
            float bamax = 0.0f;
            for (int64_t c = c0; c < c1; c++) bamax = nanmax(bamax, fabsf(load_elem(x, dtype, r * cols + c)));
            float ds = nvfp4_block_scale(bamax, gs, NULL);
            float lim = ds * 6.0f;
            for (int64_t c = c0; c < c1; c++) {
                float v = load_elem(x, dtype, r * cols + c);
                float nrm = clampf(v / ds, -6.0f, 6.0f);
                float q = round_to_e2m1(nrm, NULL) * ds;
                store_elem(y, dtype, r * cols + c, q);
                if (mask) mask[r * cols + c] = fabsf(v) <= lim;
            }
        }
    }
}

/* quantize_nvfp4 (nvfp4.py:400-462): packed u8 [rows, cols/2], E4M3 scale bytes
 * [rows, cols/16], weight_scale_2 FP32, optional reconstruction in the input dtype. */
void oracle_nvfp4_pack(const void *x, int dtype, int64_t rows, int64_t cols, float tensor_amax,
                       uint8_t *packed, uint8_t *scales, float *scale_2, void *recon) {
    int64_t nb = cols / NV_BLOCK;
    if (tensor_amax == 0.0f) { /* nvfp4.py:427-435 */
        memset(packed, 0, (size_t)(rows * cols / 2));
        memset(scales, 0x01, (size_t)(rows * nb));
        *scale_2 = 1.0f;
        if (recon) for (int64_t i = 0; i < rows * cols; i++) store_elem(recon, dtype, i, 0.0f);
        return;
    }
    float ws2 = tensor_amax / 2688.0f;
    *scale_2 = ws2;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        for (int64_t b = 0; b < nb; b++) {
            const int64_t base = r * cols + b * NV_BLOCK;
            float bamax = 0.0f;
            for (int k = 0; k < NV_BLOCK; k++) bamax = nanmax(bamax, fabsf(load_elem(x, dtype, base + k)));
            uint8_t sbyte;
            float es = nvfp4_block_scale(bamax, ws2, &sbyte);
            scales[r * nb + b] = sbyte;
            for (int k = 0; k < NV_BLOCK; k += 2) {
                uint8_t nib[2];
                for (int h = 0; h < 2; h++) {
                    float v = load_elem(x, dtype, base + k + h);
                    int idx;
                    float code = round_to_e2m1(clampf(v / es, -6.0f, 6.0f), &idx);
                    nib[h] = e2m1_nibble(code, idx);
                    if (recon) store_elem(recon, dtype, base + k + h, code * es);
                }
                packed[(base + k) / 2] = (uint8_t)((nib[0] & 0x0F) | ((nib[1] & 0x0F) << 4));
            }
        }
    }
}

/* dequantize_nvfp4 (nvfp4.py:104-121) -> FP32 */
void oracle_nvfp4_dequant(const uint8_t *packed, const uint8_t *scales, float scale_2, int64_t rows,
                          int64_t cols, float *out) {
    int64_t nb = cols / NV_BLOCK;
    for (int64_t r = 0; r < rows; r++)
        for (int64_t c = 0; c < cols; c++) {
            uint8_t byte = packed[(r * cols + c) / 2];
            uint8_t nib = (c & 1) ? (byte >> 4) : (byte & 0x0F);
            float v = E2M1_LEVELS[nib & 7];
            if (nib & 8) v = -v;
            /* weight_scale.float() is the exact E4M3 value */
            uint8_t sb = scales[r * nb + c / NV_BLOCK];
            int e = (sb >> 3) & 0x0F, m = sb & 7;
            float s = e == 0 ? (float)m * 0.001953125f : ldexpf(1.0f + (float)m / 8.0f, e - 7);
            float eff = s * scale_2;
            out[r * cols + c] = v * eff;
        }
}

/* ---------------------------------------------------------------------------- MXFP4 */

#define MX_BLOCK 32

/* 2^k built exactly for integer k in [-127, 127] */
static inline float pow2i(int k) {
    if (k == -127) return u2f(0x00400000u);
    return u2f((uint32_t)(k + 127) << 23);
}

/* _e8m0_exponent_even (mxfp4.py:48-60) */
static int e8m0_exponent_even(float block_amax) {
    int32_t bits = (int32_t)f2u(block_amax);
    uint32_t rounded = ((uint32_t)bits + 0x200000u) & 0x7F800000u;
    float rf = rounded == 0 ? u2f(0x00800000u) /* 2^-126 */ : u2f(rounded);
    float lg = floorf(log2f(rf)) - 2.0f;
    if (lg > 127.0f) lg = 127.0f;
    if (lg < -127.0f) lg = -127.0f;
    return (int)lg;
}

/* _e8m0_exponent_ceil (mxfp4.py:73-98) */
static int e8m0_exponent_ceil(float block_amax, int *zero_block) {
    float q = block_amax * 0.16666667163372039794921875f;
    uint32_t bits = f2u(q);
    int e = (int)((bits >> 23) & 0xFF);
    uint32_t man = bits & 0x7FFFFF;
    int tiny = (e == 0) && (man <= 0x400000);
    int bump = (man != 0) && !tiny;
    int biased = e + bump;
    if (biased > 254) biased = 254;
    *zero_block = biased == 0;
    return biased - 127;
}

/* _fake_quantize_mxfp4_torch (mxfp4.py:154-174), EVEN rule, zero padding to 32. */
void oracle_mxfp4_qdq_even(const void *x, int dtype, int64_t rows, int64_t cols, void *y, uint8_t *mask) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        for (int64_t c0 = 0; c0 < cols; c0 += MX_BLOCK) {
            int64_t c1 = c0 + MX_BLOCK < cols ? c0 + MX_BLOCK : cols;
            float bamax = 0.0f;
            for (int64_t c = c0; c < c1; c++) bamax = nanmax(bamax, fabsf(load_elem(x, dtype, r * cols + c)));
            float scale = pow2i(e8m0_exponent_even(bamax));
            float lim = scale * 6.0f;
            for (int64_t c = c0; c < c1; c++) {
                float v = load_elem(x, dtype, r * cols + c);
                float q = round_to_e2m1(clampf(v / scale, -6.0f, 6.0f), NULL) * scale;
                store_elem(y, dtype, r * cols + c, q);
                if (mask) mask[r * cols + c] = fabsf(v) <= lim;
            }
        }
    }
}

/* _fake_quantize_mxfp4_activation_torch (mxfp4.py:205-222), CEIL rule; cols % 32 == 0. */
void oracle_mxfp4_qdq_ceil(const void *x, int dtype, int64_t rows, int64_t cols, void *y) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        for (int64_t c0 = 0; c0 < cols; c0 += MX_BLOCK) {
            float bamax = 0.0f;
            for (int64_t c = c0; c < c0 + MX_BLOCK; c++) bamax = nanmax(bamax, fabsf(load_elem(x, dtype, r * cols + c)));
            int zero_block;
            float scale = pow2i(e8m0_exponent_ceil(bamax, &zero_block));
            for (int64_t c = c0; c < c0 + MX_BLOCK; c++) {
                float v = load_elem(x, dtype, r * cols + c);
                float q = round_to_e2m1(clampf(v / scale, -6.0f, 6.0f), NULL) * scale;
                if (zero_block) q = 0.0f;
                store_elem(y, dtype, r * cols + c, q);
            }
        }
    }
}

/* quantize_mxfp4 (mxfp4.py:126-151): packed u8 [rows, cols/2], biased E8M0 bytes
 * [rows, cols/32], optional reconstruction. */
void oracle_mxfp4_pack(const void *x, int dtype, int64_t rows, int64_t cols, uint8_t *packed,
                       uint8_t *scales, void *recon) {
    int64_t nb = cols / MX_BLOCK;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        for (int64_t b = 0; b < nb; b++) {
            const int64_t base = r * cols + b * MX_BLOCK;
            float bamax = 0.0f;
            for (int k = 0; k < MX_BLOCK; k++) bamax = nanmax(bamax, fabsf(load_elem(x, dtype, base + k)));
            int k8 = e8m0_exponent_even(bamax);
            float scale = pow2i(k8);
            scales[r * nb + b] = (uint8_t)(k8 + 127);
            for (int k = 0; k < MX_BLOCK; k += 2) {
                uint8_t nib[2];
                for (int h = 0; h < 2; h++) {
                    float v = load_elem(x, dtype, base + k + h);
                    int idx;
                    float code = round_to_e2m1(clampf(v / scale, -6.0f, 6.0f), &idx);
                    nib[h] = e2m1_nibble(code, idx);
                    if (recon) store_elem(recon, dtype, base + k + h, code * scale);
                }
                packed[(base + k) / 2] = (uint8_t)((nib[0] & 0x0F) | ((nib[1] & 0x0F) << 4));
            }
        }
    }
}

/* dequantize_mxfp4 (mxfp4.py:101-116) -> FP32 */
void oracle_mxfp4_dequant(const uint8_t *packed, const uint8_t *scales, int64_t rows, int64_t cols, float *out) {
    int64_t nb = cols / MX_BLOCK;
    for (int64_t r = 0; r < rows; r++)
        for (int64_t c = 0; c < cols; c++) {
            uint8_t byte = packed[(r * cols + c) / 2];
            uint8_t nib = (c & 1) ? (byte >> 4) : (byte & 0x0F);
            float v = E2M1_LEVELS[nib & 7];
            if (nib & 8) v = -v;
            int k = (int)scales[r * nb + c / MX_BLOCK] - 127;
            float s = pow2i(k); /* k in [-127, 128]; 128 encodes +inf like exp2 */
            out[r * cols + c] = v * s;
        }
}

/* ------------------------------------------------------------------------ STE backward */

/* _MaskedStraightThrough.backward (nvfp4.py:39-41): grad * in_range in the grad dtype. */
void oracle_ste_backward(const void *grad, int dtype, int64_t n, const uint8_t *mask, void *out) {
    for (int64_t i = 0; i < n; i++) {
        float g = load_elem(grad, dtype, i);
        store_elem(out, dtype, i, g * (mask[i] ? 1.0f : 0.0f));
    }
}

/* ----------------------------------------------------------------------------- Q4_K */

#define QK_K 256
#define Q4K_SUB 32

/* float32 sum of 32 contiguous values in torch-CPU order (see header) */
static float row_sum32(const float *v) {
    float t[8];
    for (int k = 0; k < 8; k++) t[k] = (((0.0f + v[k]) + v[k + 8]) + v[k + 16]) + v[k + 24];
    float acc = 0.0f;
    for (int k = 0; k < 8; k++) acc = acc + t[k];
    return acc;
}

static inline float fp16_round(float v) { return half_to_float(float_to_half(v)); }

/* _make_qkx2 (q4_k.py:68-119) for one 32-element sub-block; returns (scale, the_min). */
static void make_qkx2(const float *x, const float *w, float *scale_out, float *min_out) {
    const float nmax = 15.0f;
    float xmax = x[0], xmin = x[0];
    for (int i = 1; i < Q4K_SUB; i++) { xmax = nanmax(xmax, x[i]); xmin = nanmin(xmin, x[i]); }
    float vmin = clamp_max0(xmin); /* torch.minimum(min, 0) */
    int degenerate = xmax == vmin;
    float denom = degenerate ? 1.0f : xmax - vmin;
    float rden = 1.0f / denom;          /* denom.reciprocal() */
    float iscale = rden * nmax;         /* nmax / denom == reciprocal * 15 */
    float scale = (1.0f / iscale) * 1.0f;
    float xm[Q4K_SUB], prod[Q4K_SUB];
    for (int i = 0; i < Q4K_SUB; i++) xm[i] = x[i] - vmin;
    float codes;
    for (int i = 0; i < Q4K_SUB; i++) {
        codes = clampf(nearbyintf(iscale * xm[i]), 0.0f, nmax);
        float diff = ((scale * codes) + vmin) - x[i];
        prod[i] = (w[i] * diff) * diff;
    }
    float best_error = row_sum32(prod);
    float sum_w = row_sum32(w);
    for (int i = 0; i < Q4K_SUB; i++) prod[i] = w[i] * x[i];
    float sum_x = row_sum32(prod);
    float cur_min = vmin;
    for (int step = 0; step <= 20; step++) {
        /* (_RMIN + _RDELTA * step + nmax) is a Python double; torch casts it to float */
        float c = (float)(-1.0 + 0.1 * (double)step + 15.0);
        float trial_iscale = rden * c;
        float aux[Q4K_SUB], wa[Q4K_SUB], p1[Q4K_SUB], p2[Q4K_SUB];
        for (int i = 0; i < Q4K_SUB; i++) {
            aux[i] = clampf(nearbyintf(trial_iscale * xm[i]), 0.0f, nmax);
            wa[i] = w[i] * aux[i];
            p1[i] = wa[i] * aux[i];
            p2[i] = wa[i] * x[i];
        }
        float sum_l = row_sum32(wa);
        float sum_l2 = row_sum32(p1);
        float sum_xl = row_sum32(p2);
        float det = (sum_w * sum_l2) - (sum_l * sum_l);
        float safe_det = det > 0.0f ? det : 1.0f;
        float this_scale = ((sum_w * sum_xl) - (sum_x * sum_l)) / safe_det;
        float this_min = ((sum_l2 * sum_x) - (sum_l * sum_xl)) / safe_det;
        int positive_min = this_min > 0.0f;
        float safe_l2 = sum_l2 > 0.0f ? sum_l2 : 1.0f;
        if (positive_min) { this_scale = sum_xl / safe_l2; this_min = 0.0f; }
        for (int i = 0; i < Q4K_SUB; i++) {
            float d = ((this_scale * aux[i]) + this_min) - x[i];
            p1[i] = (w[i] * d) * d;
        }
        float cur_error = row_sum32(p1);
        if (det > 0.0f && cur_error < best_error) {
            best_error = cur_error;
            scale = this_scale;
            cur_min = this_min;
        }
    }
    if (degenerate) { scale = 0.0f; cur_min = vmin; }
    *scale_out = scale;
    *min_out = -cur_min;
}

/* Encode one super-block of 256 FP32 values (q4_k.py:139-207).  Writes the reconstruction
 * (FP32), the STE mask and the 144-byte block_q4_K (q4_k.py:286-337). */
static void q4k_encode_superblock(const float *xs, int method, float *recon, uint8_t *mask, uint8_t *block) {
    float scale[8], the_min[8];
    for (int j = 0; j < 8; j++) {
        const float *x = xs + j * Q4K_SUB;
        if (method == 0) { /* grid_search: _level1_grid_search_torch (q4_k.py:139-147) */
            float sq[Q4K_SUB], w[Q4K_SUB];
            for (int i = 0; i < Q4K_SUB; i++) sq[i] = x[i] * x[i];
            float av_x = sqrtf(row_sum32(sq) / 32.0f);
            for (int i = 0; i < Q4K_SUB; i++) w[i] = av_x + fabsf(x[i]);
            make_qkx2(x, w, &scale[j], &the_min[j]);
        } else { /* minmax: _level1_minmax_torch (q4_k.py:150-163) */
            float xmax = x[0], xmin = x[0];
            for (int i = 1; i < Q4K_SUB; i++) { xmax = nanmax(xmax, x[i]); xmin = nanmin(xmin, x[i]); }
            float vmin = clamp_max0(xmin); /* clamp(max=0) */
            scale[j] = (xmax - vmin) / 15.0f;
            the_min[j] = -vmin;
        }
    }
    /* _level2_encode_torch (q4_k.py:166-190) */
    float max_scale = scale[0], max_min = the_min[0];
    for (int j = 1; j < 8; j++) { max_scale = nanmax(max_scale, scale[j]); max_min = nanmax(max_min, the_min[j]); }
    float inv_scale = max_scale > 0.0f ? (1.0f / max_scale) * 63.0f : 0.0f; /* 63.0 / t */
    float inv_min = max_min > 0.0f ? (1.0f / max_min) * 63.0f : 0.0f;
    int ls[8], lm[8];
    for (int j = 0; j < 8; j++) {
        ls[j] = (int)clampf(nearbyintf(inv_scale * scale[j]), 0.0f, 63.0f);
        lm[j] = (int)clampf(nearbyintf(inv_min * the_min[j]), 0.0f, 63.0f);
    }
    uint16_t d_h = float_to_half(max_scale / 63.0f);
    uint16_t dmin_h = float_to_half(max_min / 63.0f);
    float d = half_to_float(d_h), dmin = half_to_float(dmin_h);
    uint8_t codes[QK_K];
    for (int j = 0; j < 8; j++) {
        float deff = d * (float)ls[j];
        float dm = dmin * (float)lm[j];
        int safe = deff != 0.0f;
        for (int i = 0; i < Q4K_SUB; i++) {
            int e = j * Q4K_SUB + i;
            float raw = safe ? (xs[e] + dm) / deff : 0.0f;
            float q = safe ? clampf(nearbyintf(raw), 0.0f, 15.0f) : 0.0f;
            recon[e] = (deff * q) - dm;
            mask[e] = (raw >= 0.0f) && (raw <= 15.0f);
            codes[e] = (uint8_t)q;
        }
    }
    /* [d f16][dmin f16][12 B scales][128 B qs] */
    block[0] = (uint8_t)(d_h & 0xFF); block[1] = (uint8_t)(d_h >> 8);
    block[2] = (uint8_t)(dmin_h & 0xFF); block[3] = (uint8_t)(dmin_h >> 8);
    uint8_t *s = block + 4;
    memset(s, 0, 12);
    for (int j = 0; j < 8; j++) {
        if (j < 4) {
            s[j] = (uint8_t)(ls[j] & 0x3F);
            s[j + 4] = (uint8_t)(lm[j] & 0x3F);
        } else {
            s[j + 4] = (uint8_t)((ls[j] & 0xF) | ((lm[j] & 0xF) << 4));
            s[j - 4] |= (uint8_t)((ls[j] >> 4) << 6);
            s[j] |= (uint8_t)((lm[j] >> 4) << 6);
        }
    }
    uint8_t *qs = block + 16;
    for (int g = 0; g < 4; g++)
        for (int i = 0; i < 32; i++) qs[g * 32 + i] = (uint8_t)(codes[g * 64 + i] | (codes[g * 64 + 32 + i] << 4));
}

/* quantize_q4_k / fake_quantize_q4_k (q4_k.py:245-340) over a [rows, cols] tensor with
 * cols % 256 == 0.  recon (input dtype), mask (1 byte per element) and blocks
 * ([rows, cols/256*144] bytes) may each be NULL. */
void oracle_q4k_encode(const void *x, int dtype, int64_t rows, int64_t cols, int method, void *recon,
                       uint8_t *mask, uint8_t *blocks) {
    int64_t nsb = rows * (cols / QK_K);
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t sb = 0; sb < nsb; sb++) {
        float xs[QK_K], rc[QK_K];
        uint8_t mk[QK_K], blk[144];
        for (int i = 0; i < QK_K; i++) xs[i] = load_elem(x, dtype, sb * QK_K + i);
        q4k_encode_superblock(xs, method, rc, mk, blk);
        for (int i = 0; i < QK_K; i++) {
            if (recon) store_elem(recon, dtype, sb * QK_K + i, rc[i]);
            if (mask) mask[sb * QK_K + i] = mk[i];
        }
        if (blocks) memcpy(blocks + sb * 144, blk, 144);
    }
}

/* dequantize_q4_k (q4_k.py:359-385) -> FP32 */
void oracle_q4k_dequant(const uint8_t *blocks, int64_t rows, int64_t cols, float *out) {
    int64_t nsb = rows * (cols / QK_K);
    for (int64_t sb = 0; sb < nsb; sb++) {
        const uint8_t *b = blocks + sb * 144;
        float d = half_to_float((uint16_t)(b[0] | (b[1] << 8)));
        float dmin = half_to_float((uint16_t)(b[2] | (b[3] << 8)));
        const uint8_t *s = b + 4;
        for (int j = 0; j < 8; j++) {
            int ls, lm;
            if (j < 4) { ls = s[j] & 0x3F; lm = s[j + 4] & 0x3F; }
            else { ls = (s[j + 4] & 0xF) | (((s[j - 4] >> 6) & 3) << 4); lm = (s[j + 4] >> 4) | (((s[j] >> 6) & 3) << 4); }
            float deff = d * (float)ls, dm = dmin * (float)lm;
            for (int i = 0; i < 32; i++) {
                int e = j * 32 + i;
                int g = e / 64, o = e % 64;
                uint8_t byte = b[16 + g * 32 + (o % 32)];
                int code = o < 32 ? (byte & 0xF) : (byte >> 4);
                out[sb * QK_K + e] = (deff * (float)code) - dm;
            }
        }
    }
}

/* Exposed for tests of the conversion helpers */
uint16_t oracle_float_to_bf16(float f) { return float_to_bf16(f); }
uint16_t oracle_float_to_half(float f) { return float_to_half(f); }
float oracle_cast_e4m3(float v) { return cast_e4m3(v, NULL); }
float oracle_round_to_e2m1(float v) { return round_to_e2m1(v, NULL); }

/* Level-1 fits of one FP32 super-block (tests of the encoder's intermediate values). */
void oracle_q4k_level1(const float *xs, int method, float *scale, float *the_min) {
    for (int j = 0; j < 8; j++) {
        const float *x = xs + j * Q4K_SUB;
        if (method == 0) {
            float sq[Q4K_SUB], w[Q4K_SUB];
            for (int i = 0; i < Q4K_SUB; i++) sq[i] = x[i] * x[i];
            float av_x = sqrtf(row_sum32(sq) / 32.0f);
            for (int i = 0; i < Q4K_SUB; i++) w[i] = av_x + fabsf(x[i]);
            make_qkx2(x, w, &scale[j], &the_min[j]);
        } else {
            float xmax = x[0], xmin = x[0];
            for (int i = 1; i < Q4K_SUB; i++) { xmax = nanmax(xmax, x[i]); xmin = nanmin(xmin, x[i]); }
            float vmin = clamp_max0(xmin);
            scale[j] = (xmax - vmin) / 15.0f;
            the_min[j] = -vmin;
        }
    }
}
