/*
 * kquant_scalar.c -- scalar restatement of the reference's K-quant semantics.
 * TEST INFRASTRUCTURE ONLY (see kquant_oracle.h).  Parity unpinned: no
 * runnable reference and no reference golden vectors exist for this path.
 *
 * Compiled with -ffp-contract=off: the reference's RyuJIT never fuses a*b-c
 * into an FMA on these scalar paths, and every product below is rounded on
 * its own exactly like the C# expression it restates.
 * File:line citations are relative to src/Qwen35Sharp.Kernels/.
 */
#include "kquant_oracle.h"

#include <math.h>
#include <string.h>

/* HalfBits.ToSingle (BlockLayout.cs:166): exact IEEE binary16 -> binary32,
 * subnormals included (System.Half conversion). */
float oq_fp16_to_f32(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            /* man * 2^-24 is exact in binary32 (man < 2^10). */
            float f = (float)man * 5.9604644775390625e-08f;
            memcpy(&bits, &f, 4);
            bits |= sign;
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

/* HalfBits.FromSingle (BlockLayout.cs:168): (Half)value, round to nearest
 * even.  Used only by the synthetic-input generators. */
uint16_t oq_f32_to_fp16(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0u));
    if (absx >= 0x477ff000u) /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7c00u);
    if (absx < 0x38800000u) { /* below the smallest fp16 normal: subnormal */
        if (absx < 0x33000000u) /* < 2^-25: rounds to zero (ties to even 0) */
            return (uint16_t)sign;
        uint32_t e = absx >> 23;
        uint32_t m = (absx & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126u - e; /* value = m * 2^(e-150); unit 2^-24 */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u)))
            q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (absx >> 23) - 112u;
    uint32_t m = absx & 0x7fffffu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u)))
        q++;
    return (uint16_t)(sign | q);
}

int oq_block_bytes(int type)
{
    switch (type) {
    case OQ_Q4_K: return OQ_Q4K_BYTES;
    case OQ_Q5_K: return OQ_Q5K_BYTES;
    case OQ_Q6_K: return OQ_Q6K_BYTES;
    default: return 0;
    }
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static uint32_t rd32(const uint8_t* p)
{
    uint32_t v;
    memcpy(&v, p, 4);
    return v;
}

/* ---- Q8_K ------------------------------------------------------------- */

/* Q8K.ScaleBlock, non-AVX branch (Q8K.cs:122-145): amax with the first
 * signed extremum, iscale = -127/max, delta = 1/iscale (a true reciprocal). */
static float scale_block_scalar(const float* src, float* delta)
{
    float amax = 0.f, max = 0.f;
    for (int j = 0; j < OQ_QK; j++) {
        float ax = fabsf(src[j]);
        if (ax > amax) {
            amax = ax;
            max = src[j];
        }
    }
    if (amax == 0.f) {
        *delta = 0.f;
        return 0.f;
    }
    float iscale = -127.f / max;
    *delta = 1.f / iscale;
    return iscale;
}

/* Q8K.QuantizeRow, non-AVX branches (Q8K.cs:12-77).  Output: BlockQ8K
 * (BlockLayout.cs:41-46) = f32 d, s8 qs[256], s16 bsums[16], 292 bytes. */
void oq_quantize_q8k_scalar(const float* x, void* yv, int k)
{
    uint8_t* y = (uint8_t*)yv;
    int nb = k / OQ_QK;
    for (int i = 0; i < nb; i++) {
        const float* src = x + (long)i * OQ_QK;
        uint8_t* blk = y + (long)i * OQ_Q8K_BYTES;
        float delta;
        float iscale = scale_block_scalar(src, &delta);
        if (iscale == 0.f) {
            memset(blk, 0, OQ_Q8K_BYTES);
            continue;
        }
        memcpy(blk, &delta, 4);
        int8_t* qs = (int8_t*)(blk + 4);
        for (int j = 0; j < OQ_QK; j++) {
            int v = (int)rintf(iscale * src[j]); /* MathF.Round: ties to even */
            if (v > 127) v = 127;
            if (v < -127) v = -127;
            qs[j] = (int8_t)v;
        }
        for (int j = 0; j < OQ_QK / 16; j++) {
            int sum = 0;
            for (int ii = 0; ii < 16; ii++)
                sum += qs[j * 16 + ii];
            int16_t s = (int16_t)sum;
            memcpy(blk + 260 + 2 * j, &s, 2);
        }
    }
}

/* ---- Scale unpack ------------------------------------------------------ */

/* Q4K.GetScaleMin (Q4K.cs:7-18). */
static void get_scale_min(int j, const uint8_t* s, uint8_t* sc, uint8_t* m)
{
    if (j < 4) {
        *sc = (uint8_t)(s[j] & 63);
        *m = (uint8_t)(s[j + 4] & 63);
        return;
    }
    *sc = (uint8_t)((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
    *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
}

/* Q4K.UnpackScales (Q4K.cs:20-33): bytes 0..7 = scales, 8..15 = mins. */
void oq_unpack_scales(const uint8_t* packed, uint32_t* utmp)
{
    const uint32_t kmask1 = 0x3f3f3f3fu, kmask2 = 0x0f0f0f0fu, kmask3 = 0x03030303u;
    utmp[0] = rd32(packed);
    utmp[1] = rd32(packed + 4);
    utmp[2] = rd32(packed + 8);
    utmp[3] = ((utmp[2] >> 4) & kmask2) | (((utmp[1] >> 6) & kmask3) << 4);
    uint32_t uaux = utmp[1] & kmask1;
    utmp[1] = (utmp[2] & kmask2) | (((utmp[0] >> 6) & kmask3) << 4);
    utmp[2] = uaux;
    utmp[0] &= kmask1;
}

/* ---- Dequantize -------------------------------------------------------- */

/* Q4K.DequantizeRow (Q4K.cs:35-60).  BlockQ4K = u16 d, u16 dmin,
 * u8 scales[12], u8 qs[128] (BlockLayout.cs:32-38). */
static void dequant_q4k(const uint8_t* x, float* y, int k)
{
    int nb = k / OQ_QK;
    for (int i = 0; i < nb; i++) {
        const uint8_t* b = x + (long)i * OQ_Q4K_BYTES;
        const uint8_t* q = b + 16;
        float d = oq_fp16_to_f32(rd16(b));
        float min = oq_fp16_to_f32(rd16(b + 2));
        int is = 0;
        for (int j = 0; j < OQ_QK; j += 64) {
            uint8_t sc0, m0, sc1, m1;
            get_scale_min(is + 0, b + 4, &sc0, &m0);
            get_scale_min(is + 1, b + 4, &sc1, &m1);
            float d1 = d * sc0, mm1 = min * m0;
            float d2 = d * sc1, mm2 = min * m1;
            for (int l = 0; l < 32; l++)
                *y++ = d1 * (float)(q[l] & 0xF) - mm1;
            for (int l = 0; l < 32; l++)
                *y++ = d2 * (float)(q[l] >> 4) - mm2;
            q += 32;
            is += 2;
        }
    }
}

/* Q5K.DequantizeRow (Q5K.cs:5-35).  BlockQ5K = u16 d, u16 dmin,
 * u8 scales[12], u8 qh[32], u8 qs[128] (BlockLayout.cs:49-56). */
static void dequant_q5k(const uint8_t* x, float* y, int k)
{
    int nb = k / OQ_QK;
    for (int i = 0; i < nb; i++) {
        const uint8_t* b = x + (long)i * OQ_Q5K_BYTES;
        const uint8_t* ql = b + 48;
        const uint8_t* qh = b + 16;
        float d = oq_fp16_to_f32(rd16(b));
        float min = oq_fp16_to_f32(rd16(b + 2));
        int is = 0;
        uint8_t u1 = 1, u2 = 2;
        for (int j = 0; j < OQ_QK; j += 64) {
            uint8_t sc0, m0, sc1, m1;
            get_scale_min(is + 0, b + 4, &sc0, &m0);
            get_scale_min(is + 1, b + 4, &sc1, &m1);
            float d1 = d * sc0, mm1 = min * m0;
            float d2 = d * sc1, mm2 = min * m1;
            for (int l = 0; l < 32; l++)
                *y++ = d1 * (float)((ql[l] & 0xF) + ((qh[l] & u1) ? 16 : 0)) - mm1;
            for (int l = 0; l < 32; l++)
                *y++ = d2 * (float)((ql[l] >> 4) + ((qh[l] & u2) ? 16 : 0)) - mm2;
            ql += 32;
            is += 2;
            u1 = (uint8_t)(u1 << 2);
            u2 = (uint8_t)(u2 << 2);
        }
    }
}

/* Q6K.DequantizeRow (Q6K.cs:9-39).  BlockQ6K = u8 ql[128], u8 qh[64],
 * s8 scales[16], u16 d (BlockLayout.cs:70-75). */
static void dequant_q6k(const uint8_t* x, float* y, int k)
{
    int nb = k / OQ_QK;
    for (int i = 0; i < nb; i++) {
        const uint8_t* b = x + (long)i * OQ_Q6K_BYTES;
        float d = oq_fp16_to_f32(rd16(b + 208));
        const uint8_t* ql = b;
        const uint8_t* qh = b + 128;
        const int8_t* sc = (const int8_t*)(b + 192);
        for (int n = 0; n < OQ_QK; n += 128) {
            for (int l = 0; l < 32; l++) {
                int is = l / 16;
                int q1 = (ql[l] & 0xF) | ((qh[l] & 3) << 4);
                int q2 = (ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4);
                int q3 = (ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4);
                int q4 = (ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4);
                y[l] = d * (float)sc[is] * (float)(q1 - 32);
                y[l + 32] = d * (float)sc[is + 2] * (float)(q2 - 32);
                y[l + 64] = d * (float)sc[is + 4] * (float)(q3 - 32);
                y[l + 96] = d * (float)sc[is + 6] * (float)(q4 - 32);
            }
            y += 128;
            ql += 64;
            qh += 32;
            sc += 8;
        }
    }
}

int oq_dequantize(int type, const void* blocks, float* y, int k)
{
    if (k % OQ_QK != 0)
        return -1;
    switch (type) {
    case OQ_Q4_K: dequant_q4k((const uint8_t*)blocks, y, k); return 0;
    case OQ_Q5_K: dequant_q5k((const uint8_t*)blocks, y, k); return 0;
    case OQ_Q6_K: dequant_q6k((const uint8_t*)blocks, y, k); return 0;
    default: return -1;
    }
}

/* ---- Scalar dots ------------------------------------------------------- */

static float q8_d(const uint8_t* blk)
{
    float d;
    memcpy(&d, blk, 4);
    return d;
}
static int16_t q8_bsum(const uint8_t* blk, int j)
{
    int16_t s;
    memcpy(&s, blk + 260 + 2 * j, 2);
    return s;
}

/* VecDotQ4K.DotScalar (VecDotQ4K.cs:16-65). */
static float dot_q4k_scalar(const uint8_t* x, const uint8_t* y, int n)
{
    int nb = n / OQ_QK;
    float sumf = 0.f;
    int8_t aux8[OQ_QK];
    uint32_t utmp[4];
    for (int i = 0; i < nb; i++) {
        const uint8_t* xb = x + (long)i * OQ_Q4K_BYTES;
        const uint8_t* yb = y + (long)i * OQ_Q8K_BYTES;
        const uint8_t* q4 = xb + 16;
        int8_t* a = aux8;
        for (int j = 0; j < OQ_QK / 64; j++) {
            for (int l = 0; l < 32; l++) a[l] = (int8_t)(q4[l] & 0xF);
            a += 32;
            for (int l = 0; l < 32; l++) a[l] = (int8_t)(q4[l] >> 4);
            a += 32;
            q4 += 32;
        }
        oq_unpack_scales(xb + 4, utmp);
        const uint8_t* scales = (const uint8_t*)utmp;
        const uint8_t* mins = (const uint8_t*)(utmp + 2);
        int sumi = 0;
        for (int j = 0; j < OQ_QK / 16; j++)
            sumi += q8_bsum(yb, j) * mins[j / 2];
        const int8_t* q8 = (const int8_t*)(yb + 4);
        a = aux8;
        int acc = 0;
        for (int j = 0; j < OQ_QK / 32; j++) {
            int scale = scales[j];
            for (int l = 0; l < 32; l++)
                acc += scale * q8[l] * a[l];
            q8 += 32;
            a += 32;
        }
        float d = oq_fp16_to_f32(rd16(xb)) * q8_d(yb);
        float dmin = oq_fp16_to_f32(rd16(xb + 2)) * q8_d(yb);
        sumf += d * (float)acc - dmin * (float)sumi;
    }
    return sumf;
}

/* Q5K.Dot (Q5K.cs:37-87); the reference has no SIMD variant. */
static float dot_q5k(const uint8_t* x, const uint8_t* y, int n)
{
    int nb = n / OQ_QK;
    float sumf = 0.f;
    int8_t aux[OQ_QK];
    uint32_t utmp[4];
    for (int i = 0; i < nb; i++) {
        const uint8_t* xb = x + (long)i * OQ_Q5K_BYTES;
        const uint8_t* yb = y + (long)i * OQ_Q8K_BYTES;
        const uint8_t* q4 = xb + 48;
        const uint8_t* hm = xb + 16;
        int8_t* a = aux;
        uint8_t m = 1;
        for (int j = 0; j < OQ_QK / 64; j++) {
            for (int l = 0; l < 32; l++)
                a[l] = (int8_t)((q4[l] & 0xF) + ((hm[l] & m) ? 16 : 0));
            a += 32;
            m = (uint8_t)(m << 1);
            for (int l = 0; l < 32; l++)
                a[l] = (int8_t)((q4[l] >> 4) + ((hm[l] & m) ? 16 : 0));
            a += 32;
            m = (uint8_t)(m << 1);
            q4 += 32;
        }
        oq_unpack_scales(xb + 4, utmp);
        const uint8_t* scales = (const uint8_t*)utmp;
        const uint8_t* mins = (const uint8_t*)(utmp + 2);
        int sumi = 0;
        for (int j = 0; j < OQ_QK / 16; j++)
            sumi += q8_bsum(yb, j) * mins[j / 2];
        int acc = 0;
        a = aux;
        const int8_t* q8 = (const int8_t*)(yb + 4);
        for (int j = 0; j < OQ_QK / 32; j++) {
            int scale = scales[j];
            for (int l = 0; l < 32; l++)
                acc += scale * q8[l] * a[l];
            q8 += 32;
            a += 32;
        }
        float d = oq_fp16_to_f32(rd16(xb)) * q8_d(yb);
        float dmin = oq_fp16_to_f32(rd16(xb + 2)) * q8_d(yb);
        sumf += d * (float)acc - dmin * (float)sumi;
    }
    return sumf;
}

/* Q6K.DotScalar (Q6K.cs:44-85). */
static float dot_q6k_scalar(const uint8_t* x, const uint8_t* y, int n)
{
    int nb = n / OQ_QK;
    float sumf = 0.f;
    int8_t aux[OQ_QK];
    for (int i = 0; i < nb; i++) {
        const uint8_t* xb = x + (long)i * OQ_Q6K_BYTES;
        const uint8_t* yb = y + (long)i * OQ_Q8K_BYTES;
        const uint8_t* q4 = xb;
        const uint8_t* qh = xb + 128;
        int8_t* a = aux;
        for (int j = 0; j < OQ_QK; j += 128) {
            for (int l = 0; l < 32; l++) {
                a[l] = (int8_t)(((q4[l] & 0xF) | ((qh[l] & 3) << 4)) - 32);
                a[l + 32] = (int8_t)(((q4[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32);
                a[l + 64] = (int8_t)(((q4[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32);
                a[l + 96] = (int8_t)(((q4[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32);
            }
            a += 128;
            q4 += 64;
            qh += 32;
        }
        int acc = 0;
        a = aux;
        const int8_t* q8 = (const int8_t*)(yb + 4);
        const int8_t* sc = (const int8_t*)(xb + 192);
        for (int j = 0; j < OQ_QK / 16; j++) {
            int scale = sc[j];
            for (int l = 0; l < 16; l++)
                acc += scale * q8[l] * a[l];
            q8 += 16;
            a += 16;
        }
        sumf += oq_fp16_to_f32(rd16(xb + 208)) * q8_d(yb) * (float)acc;
    }
    return sumf;
}

float oq_dot_scalar(int type, const void* w, const void* q8, int n)
{
    switch (type) {
    case OQ_Q4_K: return dot_q4k_scalar((const uint8_t*)w, (const uint8_t*)q8, n);
    case OQ_Q5_K: return dot_q5k((const uint8_t*)w, (const uint8_t*)q8, n);
    case OQ_Q6_K: return dot_q6k_scalar((const uint8_t*)w, (const uint8_t*)q8, n);
    default: return NAN;
    }
}

/* ---- Panel GEMM semantics --------------------------------------------- */

/* GemmQ4K.GemmScalar (GemmQ4K.cs:25-106) restated on row-major Q4_K blocks
 * instead of the BlockQ4Kx8 panel (same values, same fp32 operation order):
 * per 16-value k-step, sumi = sum of 8 low-nibble and 8 high-nibble products
 * times their sub-block scales, dest += sumi * d_col * d_row (AddCol,
 * :126-141); mins once per 32-value sub-block (AccumulateMins, :144-160),
 * output = s - m (:92-103). */
void oq_gemm_q4k_semantic(const void* wv, const void* q8v, float* dst, int ldc,
                          int nIn, int rows, int cols)
{
    const uint8_t* w = (const uint8_t*)wv;
    const uint8_t* q8 = (const uint8_t*)q8v;
    int nb = nIn / OQ_QK;
    for (int r = 0; r < rows; r++) {
        for (int c = 0; c < cols; c++) {
            float s = 0.f, mm = 0.f;
            for (int l = 0; l < nb; l++) {
                const uint8_t* b = w + ((long)c * nb + l) * OQ_Q4K_BYTES;
                const uint8_t* a = q8 + ((long)r * nb + l) * OQ_Q8K_BYTES;
                const int8_t* aq = (const int8_t*)(a + 4);
                uint8_t sc[8], mn[8];
                for (int j = 0; j < 8; j++)
                    get_scale_min(j, b + 4, &sc[j], &mn[j]);
                float dcol = oq_fp16_to_f32(rd16(b));
                float dmincol = oq_fp16_to_f32(rd16(b + 2));
                float ad = q8_d(a);
                for (int k = 0; k < 16; k++) {
                    int g = k / 4, st = k % 4;
                    int sumi = 0;
                    for (int i = 0; i < 8; i++) {
                        int pos = 64 * g + 8 * st + i;
                        int byte = b[16 + 32 * g + 8 * st + i];
                        sumi += (byte & 0xF) * aq[pos] * sc[2 * g];
                        sumi += (byte >> 4) * aq[pos + 32] * sc[2 * g + 1];
                    }
                    s += (float)sumi * dcol * ad;
                }
                for (int sb = 0; sb < 8; sb++) {
                    int pair = q8_bsum(a, 2 * sb) + q8_bsum(a, 2 * sb + 1);
                    mm += (float)(mn[sb] * pair) * dmincol * ad;
                }
            }
            dst[(long)r * ldc + c] = s - mm;
        }
    }
}
