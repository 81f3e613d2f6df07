/*
 * kquant_avx2.c -- AVX2 restatement of the instruction sequences the
 * reference executes on x86 with AVX2+FMA, plus its threaded dispatch.
 * TEST INFRASTRUCTURE ONLY (see kquant_oracle.h); this is the timed CPU
 * baseline ("port" of the reference kernels).  Parity unpinned: no runnable
 * reference and no reference golden vectors exist for this path.
 *
 * Built with -O2 -mavx2 -mfma -mf16c -ffp-contract=off: FMAs appear only
 * where the reference calls Fma.MultiplyAdd explicitly.
 * File:line citations are relative to src/Qwen35Sharp.Kernels/.
 */
#define _GNU_SOURCE
#include "kquant_oracle.h"

#include <immintrin.h>
#include <pthread.h>
#include <sched.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

void oq_unpack_scales(const uint8_t* packed, uint32_t* utmp);

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static float q8_d(const uint8_t* blk)
{
    float d;
    memcpy(&d, blk, 4);
    return d;
}

/* VecDotQ4K.HorizontalSum (VecDotQ4K.cs:144-151). */
static inline float hsum256(__m256 v)
{
    __m128 s = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
    s = _mm_add_ps(s, _mm_movehl_ps(s, s));
    s = _mm_add_ss(s, _mm_shuffle_ps(s, s, 0x55));
    return _mm_cvtss_f32(s);
}

/* ---- Q8_K (AVX2 branches) --------------------------------------------- */

/* Q8K.ScaleBlock, AVX branch (Q8K.cs:87-121, 143-145). */
static float scale_block_avx(const float* src, float* delta)
{
    __m256 vacc = _mm256_setzero_ps();
    __m256 sign = _mm256_set1_ps(-0.0f);
    for (int j = 0; j < OQ_QK; j += 8)
        vacc = _mm256_max_ps(vacc, _mm256_andnot_ps(sign, _mm256_loadu_ps(src + j)));
    __m128 lane = _mm_max_ps(_mm256_castps256_ps128(vacc), _mm256_extractf128_ps(vacc, 1));
    lane = _mm_max_ps(lane, _mm_movehl_ps(lane, lane));
    lane = _mm_max_ps(lane, _mm_shuffle_ps(lane, lane, 0x55));
    float amax = _mm_cvtss_f32(lane);
    if (amax == 0.f) {
        *delta = 0.f;
        return 0.f;
    }
    __m256 pos = _mm256_set1_ps(amax), neg = _mm256_set1_ps(-amax);
    int first_pos = OQ_QK, first_neg = OQ_QK;
    for (int j = 0; j < OQ_QK; j += 8) {
        __m256 v = _mm256_loadu_ps(src + j);
        int mp = _mm256_movemask_ps(_mm256_cmp_ps(v, pos, _CMP_EQ_OQ));
        int mn = _mm256_movemask_ps(_mm256_cmp_ps(v, neg, _CMP_EQ_OQ));
        if (mp && j + __builtin_ctz(mp) < first_pos) first_pos = j + __builtin_ctz(mp);
        if (mn && j + __builtin_ctz(mn) < first_neg) first_neg = j + __builtin_ctz(mn);
        if ((first_pos < first_neg ? first_pos : first_neg) < j + 8)
            break;
    }
    float max = first_neg < first_pos ? -amax : amax;
    float iscale = -127.f / max;
    *delta = 1.f / iscale;
    return iscale;
}

/* Q8K.QuantizeRow, AVX2 branches (Q8K.cs:29-41, 54-65). */
void oq_quantize_q8k_avx2(const float* x, void* yv, int k)
{
    uint8_t* y = (uint8_t*)yv;
    int nb = k / OQ_QK;
    for (int i = 0; i < nb; i++) {
        const float* src = x + (long)i * OQ_QK;
        uint8_t* blk = y + (long)i * OQ_Q8K_BYTES;
        float delta;
        float iscale = scale_block_avx(src, &delta);
        if (iscale == 0.f) {
            memset(blk, 0, OQ_Q8K_BYTES);
            continue;
        }
        memcpy(blk, &delta, 4);
        int8_t* qs = (int8_t*)(blk + 4);
        __m256 isv = _mm256_set1_ps(iscale);
        __m256i lo = _mm256_set1_epi32(-127), hi = _mm256_set1_epi32(127);
        for (int j = 0; j < OQ_QK; j += 8) {
            __m256 r = _mm256_round_ps(_mm256_mul_ps(_mm256_loadu_ps(src + j), isv),
                                       _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
            __m256i qi = _mm256_min_epi32(_mm256_max_epi32(_mm256_cvtps_epi32(r), lo), hi);
            __m128i p16 = _mm_packs_epi32(_mm256_castsi256_si128(qi), _mm256_extracti128_si256(qi, 1));
            __m128i p8 = _mm_packs_epi16(p16, _mm_setzero_si128());
            _mm_storel_epi64((__m128i*)(qs + j), p8);
        }
        for (int j = 0; j < OQ_QK / 16; j++) {
            __m256i w = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(qs + j * 16)));
            __m128i s = _mm_hadd_epi16(_mm256_castsi256_si128(w), _mm256_extracti128_si256(w, 1));
            s = _mm_hadd_epi16(s, s);
            s = _mm_hadd_epi16(s, s);
            s = _mm_hadd_epi16(s, s);
            int16_t v = (int16_t)_mm_cvtsi128_si32(s);
            memcpy(blk + 260 + 2 * j, &v, 2);
        }
    }
}

/* ---- Q4_K dot (VecDotQ4K.DotAvx2, VecDotQ4K.cs:67-126) ----------------- */

static inline __m256i scale_shuffle_q4(int i)
{
    /* ScaleShuffle (VecDotQ4K.cs:128-142): broadcast int16 element i. */
    return _mm256_set1_epi16((short)((2 * i) | ((2 * i + 1) << 8)));
}

static float dot_q4k_avx2(const uint8_t* x, const uint8_t* y, int n)
{
    int nb = n / OQ_QK;
    uint32_t utmp[4];
    const __m256i m4 = _mm256_set1_epi8(0x0F);
    __m256 acc = _mm256_setzero_ps();
    __m128 acc_min = _mm_setzero_ps();
    for (int i = 0; i < nb; i++) {
        const uint8_t* xb = x + (long)i * OQ_Q4K_BYTES;
        const uint8_t* yb = y + (long)i * OQ_Q8K_BYTES;
        float yd = q8_d(yb);
        float d = yd * oq_fp16_to_f32(rd16(xb));
        float dmin = -yd * oq_fp16_to_f32(rd16(xb + 2));
        oq_unpack_scales(xb + 4, utmp);
        const uint8_t* q4 = xb + 16;
        const int8_t* q8 = (const int8_t*)(yb + 4);

        __m128i packed = _mm_loadu_si128((const __m128i*)utmp);
        __m256i mins_and_scales = _mm256_cvtepu8_epi16(packed);
        __m256i q8sums = _mm256_loadu_si256((const __m256i*)(yb + 260));
        __m128i q8s = _mm_hadd_epi16(_mm256_castsi256_si128(q8sums), _mm256_extracti128_si256(q8sums, 1));
        __m128i prod = _mm_madd_epi16(_mm256_extracti128_si256(mins_and_scales, 1), q8s);
        acc_min = _mm_add_ps(acc_min, _mm_mul_ps(_mm_set1_ps(dmin), _mm_cvtepi32_ps(prod)));

        __m128i sc128 = _mm256_castsi256_si128(mins_and_scales);
        __m256i scales = _mm256_set_m128i(sc128, sc128);
        __m256i sumi = _mm256_setzero_si256();
        for (int j = 0; j < OQ_QK / 64; j++) {
            __m256i scale_l = _mm256_shuffle_epi8(scales, scale_shuffle_q4(2 * j + 0));
            __m256i scale_h = _mm256_shuffle_epi8(scales, scale_shuffle_q4(2 * j + 1));
            __m256i q4bits = _mm256_loadu_si256((const __m256i*)q4);
            q4 += 32;
            __m256i q4l = _mm256_and_si256(q4bits, m4);
            __m256i q4h = _mm256_and_si256(_mm256_srli_epi16(q4bits, 4), m4);
            __m256i q8l = _mm256_loadu_si256((const __m256i*)q8);
            q8 += 32;
            __m256i p32l = _mm256_madd_epi16(_mm256_maddubs_epi16(q4l, q8l), scale_l);
            __m256i q8h = _mm256_loadu_si256((const __m256i*)q8);
            q8 += 32;
            __m256i p32h = _mm256_madd_epi16(_mm256_maddubs_epi16(q4h, q8h), scale_h);
            sumi = _mm256_add_epi32(sumi, _mm256_add_epi32(p32l, p32h));
        }
        acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(sumi), _mm256_set1_ps(d), acc);
    }
    acc_min = _mm_add_ps(acc_min, _mm_movehl_ps(acc_min, acc_min));
    acc_min = _mm_add_ss(acc_min, _mm_shuffle_ps(acc_min, acc_min, 0x55));
    return hsum256(acc) + _mm_cvtss_f32(acc_min);
}

/* ---- Q6_K dots (Q6K.DotAvx2 :87-167, Q6K.DotAvx2x4 :172-248) ------------ */

static inline __m128i scale_shuffle_q6(int i)
{
    /* ScaleShuffle + ScaleShuffleBytes (Q6K.cs:283-299): bytes 2i x8 then 2i+1 x8. */
    return _mm_set_epi64x((long long)(0x0101010101010101ULL * (uint64_t)(2 * i + 1)),
                          (long long)(0x0101010101010101ULL * (uint64_t)(2 * i)));
}

typedef struct {
    __m256i q40, q41, q42, q43;
} q6_quads;

static inline q6_quads q6_decode(const uint8_t* ql, const uint8_t* qh)
{
    const __m256i m3 = _mm256_set1_epi8(3), m15 = _mm256_set1_epi8(15);
    const __m256i m12 = _mm256_set1_epi8(12), m48 = _mm256_set1_epi8(48);
    const __m256i mc0 = _mm256_set1_epi8((char)0xC0);
    __m256i b1 = _mm256_loadu_si256((const __m256i*)ql);
    __m256i b2 = _mm256_loadu_si256((const __m256i*)(ql + 32));
    __m256i bh = _mm256_loadu_si256((const __m256i*)qh);
    __m256i h0 = _mm256_slli_epi16(_mm256_and_si256(bh, m3), 4);
    __m256i h1 = _mm256_slli_epi16(_mm256_and_si256(bh, m12), 2);
    __m256i h2 = _mm256_and_si256(bh, m48);
    __m256i h3 = _mm256_srli_epi16(_mm256_and_si256(bh, mc0), 2);
    q6_quads q;
    q.q40 = _mm256_or_si256(_mm256_and_si256(b1, m15), h0);
    q.q41 = _mm256_or_si256(_mm256_and_si256(b2, m15), h1);
    q.q42 = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(b1, 4), m15), h2);
    q.q43 = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(b2, 4), m15), h3);
    return q;
}

static float dot_q6k_avx2(const uint8_t* x, const uint8_t* y, int n)
{
    int nb = n / OQ_QK;
    __m256 acc = _mm256_setzero_ps();
    for (int i = 0; i < nb; i++) {
        const uint8_t* xb = x + (long)i * OQ_Q6K_BYTES;
        const uint8_t* yb = y + (long)i * OQ_Q8K_BYTES;
        float d = q8_d(yb) * oq_fp16_to_f32(rd16(xb + 208));
        const uint8_t* q4 = xb;
        const uint8_t* qh = xb + 128;
        const int8_t* q8 = (const int8_t*)(yb + 4);
        __m256i q8sums = _mm256_loadu_si256((const __m256i*)(yb + 260));
        __m128i scales = _mm_loadu_si128((const __m128i*)(xb + 192));
        __m256i scales16 = _mm256_cvtepi8_epi16(scales);
        __m256i q8sclsub = _mm256_slli_epi32(_mm256_madd_epi16(q8sums, scales16), 5);
        __m256i sumi = _mm256_setzero_si256();
        int is = 0;
        for (int j = 0; j < OQ_QK / 128; j++) {
            q6_quads q = q6_decode(q4, qh);
            q4 += 64;
            qh += 32;
            __m256i p0 = _mm256_maddubs_epi16(q.q40, _mm256_loadu_si256((const __m256i*)(q8 + 0)));
            __m256i p1 = _mm256_maddubs_epi16(q.q41, _mm256_loadu_si256((const __m256i*)(q8 + 32)));
            __m256i p2 = _mm256_maddubs_epi16(q.q42, _mm256_loadu_si256((const __m256i*)(q8 + 64)));
            __m256i p3 = _mm256_maddubs_epi16(q.q43, _mm256_loadu_si256((const __m256i*)(q8 + 96)));
            q8 += 128;
            __m256i i0 = _mm256_madd_epi16(_mm256_cvtepi8_epi16(_mm_shuffle_epi8(scales, scale_shuffle_q6(is + 0))), p0);
            __m256i i1 = _mm256_madd_epi16(_mm256_cvtepi8_epi16(_mm_shuffle_epi8(scales, scale_shuffle_q6(is + 1))), p1);
            __m256i i2 = _mm256_madd_epi16(_mm256_cvtepi8_epi16(_mm_shuffle_epi8(scales, scale_shuffle_q6(is + 2))), p2);
            __m256i i3 = _mm256_madd_epi16(_mm256_cvtepi8_epi16(_mm_shuffle_epi8(scales, scale_shuffle_q6(is + 3))), p3);
            is += 4;
            sumi = _mm256_add_epi32(sumi, _mm256_add_epi32(i0, i1));
            sumi = _mm256_add_epi32(sumi, _mm256_add_epi32(i2, i3));
        }
        sumi = _mm256_sub_epi32(sumi, q8sclsub);
        acc = _mm256_fmadd_ps(_mm256_set1_ps(d), _mm256_cvtepi32_ps(sumi), acc);
    }
    return hsum256(acc);
}

void oq_dot_q6k_avx2x4(const void* wv, const void* y0v, const void* y1v,
                       const void* y2v, const void* y3v, int n, float* dst)
{
    const uint8_t* x = (const uint8_t*)wv;
    const uint8_t* ys[4] = {(const uint8_t*)y0v, (const uint8_t*)y1v, (const uint8_t*)y2v, (const uint8_t*)y3v};
    int nb = n / OQ_QK;
    __m256 acc[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
    for (int i = 0; i < nb; i++) {
        const uint8_t* xb = x + (long)i * OQ_Q6K_BYTES;
        float xd = oq_fp16_to_f32(rd16(xb + 208));
        const uint8_t* q4 = xb;
        const uint8_t* qh = xb + 128;
        __m128i scales = _mm_loadu_si128((const __m128i*)(xb + 192));
        __m256i scales16 = _mm256_cvtepi8_epi16(scales);
        __m256i sum[4] = {_mm256_setzero_si256(), _mm256_setzero_si256(), _mm256_setzero_si256(), _mm256_setzero_si256()};
        int is = 0;
        for (int j = 0; j < OQ_QK / 128; j++) {
            q6_quads q = q6_decode(q4, qh);
            q4 += 64;
            qh += 32;
            __m256i sc0 = _mm256_cvtepi8_epi16(_mm_shuffle_epi8(scales, scale_shuffle_q6(is + 0)));
            __m256i sc1 = _mm256_cvtepi8_epi16(_mm_shuffle_epi8(scales, scale_shuffle_q6(is + 1)));
            __m256i sc2 = _mm256_cvtepi8_epi16(_mm_shuffle_epi8(scales, scale_shuffle_q6(is + 2)));
            __m256i sc3 = _mm256_cvtepi8_epi16(_mm_shuffle_epi8(scales, scale_shuffle_q6(is + 3)));
            is += 4;
            for (int t = 0; t < 4; t++) {
                /* AccumulateQ6Lane (Q6K.cs:251-272) */
                const int8_t* q8 = (const int8_t*)(ys[t] + (long)i * OQ_Q8K_BYTES + 4) + j * 128;
                __m256i p0 = _mm256_maddubs_epi16(q.q40, _mm256_loadu_si256((const __m256i*)q8));
                __m256i p1 = _mm256_maddubs_epi16(q.q41, _mm256_loadu_si256((const __m256i*)(q8 + 32)));
                __m256i p2 = _mm256_maddubs_epi16(q.q42, _mm256_loadu_si256((const __m256i*)(q8 + 64)));
                __m256i p3 = _mm256_maddubs_epi16(q.q43, _mm256_loadu_si256((const __m256i*)(q8 + 96)));
                __m256i i0 = _mm256_madd_epi16(sc0, p0);
                __m256i i1 = _mm256_madd_epi16(sc1, p1);
                __m256i i2 = _mm256_madd_epi16(sc2, p2);
                __m256i i3 = _mm256_madd_epi16(sc3, p3);
                sum[t] = _mm256_add_epi32(sum[t], _mm256_add_epi32(_mm256_add_epi32(i0, i1), _mm256_add_epi32(i2, i3)));
            }
        }
        for (int t = 0; t < 4; t++) {
            const uint8_t* yb = ys[t] + (long)i * OQ_Q8K_BYTES;
            __m256i sub = _mm256_slli_epi32(_mm256_madd_epi16(_mm256_loadu_si256((const __m256i*)(yb + 260)), scales16), 5);
            sum[t] = _mm256_sub_epi32(sum[t], sub);
            /* MaddScale (Q6K.cs:275-280) with d = xd * y.D */
            acc[t] = _mm256_fmadd_ps(_mm256_set1_ps(xd * q8_d(yb)), _mm256_cvtepi32_ps(sum[t]), acc[t]);
        }
    }
    for (int t = 0; t < 4; t++)
        dst[t] = hsum256(acc[t]);
}

float oq_dot_avx2(int type, const void* w, const void* q8, int n)
{
    switch (type) {
    case OQ_Q4_K: return dot_q4k_avx2((const uint8_t*)w, (const uint8_t*)q8, n);
    case OQ_Q5_K: return oq_dot_scalar(OQ_Q5_K, w, q8, n); /* Q5K.Dot is scalar only */
    case OQ_Q6_K: return dot_q6k_avx2((const uint8_t*)w, (const uint8_t*)q8, n);
    default: return 0.f;
    }
}

/* ---- Q8_Kx4 and the Q4_K panel ----------------------------------------- */

static int16_t sum8(const int8_t* p)
{
    int s = 0;
    for (int i = 0; i < 8; i++) s += p[i];
    return (int16_t)s;
}

/* QuantizeQ8Kx4.Quantize4x8Avx2 (QuantizeQ8Kx4.cs:108-144) and FillBsums
 * (:191-203).  BlockQ8Kx4 = f32 d[4], s8 qs[1024] (8-byte chunks of the 4
 * rows interleaved), s16 bsums[64] (BlockLayout.cs:141-146). */
void oq_quantize_q8kx4(const float* x, void* yv, int k)
{
    uint8_t* y = (uint8_t*)yv;
    int nb = k / OQ_QK;
    const __m256i perm = _mm256_setr_epi32(0, 4, 1, 5, 2, 6, 3, 7);
    const __m256i qmin = _mm256_set1_epi32(-127), qmax = _mm256_set1_epi32(127);
    for (int i = 0; i < nb; i++) {
        uint8_t* blk = y + (long)i * OQ_Q8KX4_BYTES;
        float is[4], d[4];
        for (int r = 0; r < 4; r++)
            is[r] = scale_block_avx(x + (long)r * k + (long)i * OQ_QK, &d[r]);
        memcpy(blk, d, 16);
        int8_t* qs = (int8_t*)(blk + 16);
        for (int j = 0; j < 32; j++) {
            __m256i v[4];
            for (int r = 0; r < 4; r++) {
                /* Quant8 (QuantizeQ8Kx4.cs:184-188) */
                __m256 rr = _mm256_round_ps(_mm256_mul_ps(_mm256_loadu_ps(x + (long)r * k + (long)i * OQ_QK + j * 8),
                                                          _mm256_set1_ps(is[r])),
                                            _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
                v[r] = _mm256_min_epi32(_mm256_max_epi32(_mm256_cvtps_epi32(rr), qmin), qmax);
            }
            __m256i p01 = _mm256_packs_epi32(v[0], v[1]);
            __m256i p23 = _mm256_packs_epi32(v[2], v[3]);
            __m256i packed = _mm256_permutevar8x32_epi32(_mm256_packs_epi16(p01, p23), perm);
            _mm256_storeu_si256((__m256i*)(qs + 32 * j), packed);
        }
        int16_t* bsums = (int16_t*)(blk + 16 + 1024);
        for (int t = 0; t < OQ_QK / 16; t++) {
            int dest = ((t >> 2) << 4) + (t & 3);
            int c0 = (t * 2) * 32, c1 = c0 + 32;
            for (int r = 0; r < 4; r++) {
                int16_t s = (int16_t)(sum8(qs + c0 + 8 * r) + sum8(qs + c1 + 8 * r));
                memcpy(&bsums[dest + 4 * r], &s, 2);
            }
        }
    }
}

static void get_scale_min(int j, const uint8_t* q, uint8_t* d, uint8_t* m)
{
    if (j < 4) {
        *d = (uint8_t)(q[j] & 63);
        *m = (uint8_t)(q[j + 4] & 63);
    } else {
        *d = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* RepackQ4K.MakeBlockX8 qs interleave (RepackQ4K.cs:5-21) via Rows (:71-85).
 * Only the fields the AVX2 GEMM reads are produced: D/Dmin (fp16) and the
 * 8-byte interleaved qs; the packed 6-bit scales feed GemmScalar only, whose
 * semantics oq_gemm_q4k_semantic restates on row-major blocks. */
void oq_repack_q4kx8(const void* srcv, void* dstv, int nIn, int nOut)
{
    const uint8_t* src = (const uint8_t*)srcv;
    uint8_t* dst = (uint8_t*)dstv;
    int nb = nIn / OQ_QK, groups = nOut / 8;
    for (int g = 0; g < groups; g++) {
        for (int b = 0; b < nb; b++) {
            uint8_t* out = dst + ((long)g * nb + b) * OQ_Q4KX8_BYTES;
            memset(out, 0, OQ_Q4KX8_BYTES);
            for (int r = 0; r < 8; r++) {
                const uint8_t* in = src + ((long)(g * 8 + r) * nb + b) * OQ_Q4K_BYTES;
                memcpy(out + 2 * r, in, 2);
                memcpy(out + 16 + 2 * r, in + 2, 2);
            }
            for (int i = 0; i < OQ_QK * 4 / 8; i++) {
                int sid = i % 8, soff = (i / 8) * 8;
                const uint8_t* in = src + ((long)(g * 8 + sid) * nb + b) * OQ_Q4K_BYTES;
                memcpy(out + 128 + i * 8, in + 16 + soff, 8);
            }
        }
    }
}

/* RepackQ4K.BuildMeta (RepackQ4K.cs:91-130): f32 d[8], f32 dmin[8], then per
 * 64-value pair: lo scales, hi scales in vphaddw order, mins interleaved. */
void oq_build_meta_q4kx8(const void* srcv, void* dstv, int nIn, int nOut)
{
    static const int order[16] = {0, 0, 1, 1, 4, 4, 5, 5, 2, 2, 3, 3, 6, 6, 7, 7};
    const uint8_t* src = (const uint8_t*)srcv;
    uint8_t* dst = (uint8_t*)dstv;
    int nb = nIn / OQ_QK, groups = nOut / 8;
    for (int g = 0; g < groups; g++) {
        for (int b = 0; b < nb; b++) {
            uint8_t* meta = dst + ((long)g * nb + b) * OQ_Q4KX8_META_BYTES;
            float* md = (float*)meta;
            float* mdm = (float*)(meta + 32);
            int16_t* msc = (int16_t*)(meta + 64);
            for (int j = 0; j < 8; j++) {
                const uint8_t* blk = src + ((long)(g * 8 + j) * nb + b) * OQ_Q4K_BYTES;
                md[j] = oq_fp16_to_f32(rd16(blk));
                mdm[j] = oq_fp16_to_f32(rd16(blk + 2));
            }
            for (int pair = 0; pair < 4; pair++) {
                int16_t* lo = msc + pair * 48;
                int16_t* hi = lo + 16;
                int16_t* mins = lo + 32;
                for (int half = 0; half < 2; half++) {
                    uint8_t sc[8], mn[8];
                    int sub = pair * 2 + half;
                    for (int j = 0; j < 8; j++)
                        get_scale_min(sub, src + ((long)(g * 8 + j) * nb + b) * OQ_Q4K_BYTES + 4, &sc[j], &mn[j]);
                    int16_t* target = half == 0 ? lo : hi;
                    for (int i = 0; i < 16; i++)
                        target[i] = sc[order[i]];
                    for (int j = 0; j < 8; j++)
                        mins[j * 2 + half] = mn[j];
                }
            }
        }
    }
}

/* GemmQ4K.RowSum (GemmQ4K.Avx2.cs:212-213). */
static inline __m256 row_sum(__m256i a0123, __m256i a4567, __m256i scales)
{
    return _mm256_cvtepi32_ps(_mm256_madd_epi16(_mm256_hadd_epi16(a0123, a4567), scales));
}

/* GemmQ4K.GemmAvx2Tile (GemmQ4K.Avx2.cs:39-205). */
static void gemm_avx2_tile(int n, float* dst, int ldc, const uint8_t* weights,
                           const uint8_t* acts, int rows, int cols, const uint8_t* meta_base)
{
    int nb = n / OQ_QK;
    const __m256i m4b = _mm256_set1_epi8(0x0F);
    const __m256i col_perm = _mm256_setr_epi32(0, 1, 4, 5, 2, 3, 6, 7);
    for (int yy = 0; yy < rows / 4; yy++) {
        const uint8_t* a_ptr = acts + (long)yy * nb * OQ_Q8KX4_BYTES;
        for (int xx = 0; xx < cols / 8; xx++) {
            const uint8_t* b_ptr = weights + (long)xx * nb * OQ_Q4KX8_BYTES;
            const uint8_t* meta = meta_base + (long)xx * nb * OQ_Q4KX8_META_BYTES;
            __m256 acc[4], mn[4];
            for (int r = 0; r < 4; r++) {
                acc[r] = _mm256_setzero_ps();
                mn[r] = _mm256_setzero_ps();
            }
            for (int b = 0; b < nb; b++) {
                const uint8_t* mb = meta + (long)b * OQ_Q4KX8_META_BYTES;
                const uint8_t* ab = a_ptr + (long)b * OQ_Q8KX4_BYTES;
                __m256 col_scale = _mm256_permutevar8x32_ps(_mm256_loadu_ps((const float*)mb), col_perm);
                __m128 rs4 = _mm_loadu_ps((const float*)ab);
                __m256 row_scale = _mm256_set_m128(rs4, rs4);
                __m256 cs[4];
                cs[0] = _mm256_mul_ps(col_scale, _mm256_shuffle_ps(row_scale, row_scale, 0));
                cs[1] = _mm256_mul_ps(col_scale, _mm256_shuffle_ps(row_scale, row_scale, 85));
                cs[2] = _mm256_mul_ps(col_scale, _mm256_shuffle_ps(row_scale, row_scale, 170));
                cs[3] = _mm256_mul_ps(col_scale, _mm256_shuffle_ps(row_scale, row_scale, 255));
                const uint8_t* qs = b_ptr + (long)b * OQ_Q4KX8_BYTES + 128;
                const uint8_t* aqs = ab + 16;
                const int16_t* sc = (const int16_t*)(mb + 64);
                for (int sb = 0; sb < OQ_QK / 64; sb++) {
                    for (int half = 0; half < 2; half++) {
                        /* half 0: low nibbles = sub-block 2*sb; half 1: high. */
                        const uint8_t* q = qs;
                        const int64_t* a = (const int64_t*)(aqs + half * 128);
                        __m256i ia[4], ib[4];
                        for (int s = 0; s < 4; s++) {
                            __m256i r0123 = _mm256_loadu_si256((const __m256i*)q);
                            __m256i r4567 = _mm256_loadu_si256((const __m256i*)(q + 32));
                            if (half) {
                                r0123 = _mm256_srli_epi16(r0123, 4);
                                r4567 = _mm256_srli_epi16(r4567, 4);
                            }
                            r0123 = _mm256_and_si256(r0123, m4b);
                            r4567 = _mm256_and_si256(r4567, m4b);
                            for (int r = 0; r < 4; r++) {
                                int64_t av;
                                memcpy(&av, a + r, 8);
                                __m256i l = _mm256_set1_epi64x(av);
                                __m256i pa = _mm256_maddubs_epi16(r0123, l);
                                __m256i pb = _mm256_maddubs_epi16(r4567, l);
                                ia[r] = s == 0 ? pa : _mm256_add_epi16(ia[r], pa);
                                ib[r] = s == 0 ? pb : _mm256_add_epi16(ib[r], pb);
                            }
                            q += 64;
                            a += 4;
                        }
                        __m256i scv = _mm256_loadu_si256((const __m256i*)(sc + 16 * half));
                        for (int r = 0; r < 4; r++)
                            acc[r] = _mm256_fmadd_ps(row_sum(ia[r], ib[r], scv), cs[r], acc[r]);
                    }
                    qs += 256;
                    aqs += 256;
                    sc += 48;
                }
                /* dmin compensation once per super-block (:171-196). */
                __m256i m[4] = {_mm256_setzero_si256(), _mm256_setzero_si256(), _mm256_setzero_si256(), _mm256_setzero_si256()};
                const int16_t* bs = (const int16_t*)(ab + 16 + 1024);
                const int16_t* mins = (const int16_t*)(mb + 64) + 32;
                for (int p = 0; p < 4; p++) {
                    __m256i bsums = _mm256_loadu_si256((const __m256i*)bs);
                    __m128i bsum_h = _mm_hadd_epi16(_mm256_castsi256_si128(bsums), _mm256_extracti128_si256(bsums, 1));
                    __m256i dup = _mm256_set_m128i(bsum_h, bsum_h);
                    __m256i mins01 = _mm256_loadu_si256((const __m256i*)mins);
                    m[0] = _mm256_add_epi32(m[0], _mm256_madd_epi16(_mm256_shuffle_epi32(dup, 0), mins01));
                    m[1] = _mm256_add_epi32(m[1], _mm256_madd_epi16(_mm256_shuffle_epi32(dup, 85), mins01));
                    m[2] = _mm256_add_epi32(m[2], _mm256_madd_epi16(_mm256_shuffle_epi32(dup, 170), mins01));
                    m[3] = _mm256_add_epi32(m[3], _mm256_madd_epi16(_mm256_shuffle_epi32(dup, 255), mins01));
                    bs += 16;
                    mins += 48;
                }
                __m256 col_dmin = _mm256_loadu_ps((const float*)(mb + 32));
                mn[0] = _mm256_fmadd_ps(_mm256_cvtepi32_ps(m[0]), _mm256_mul_ps(col_dmin, _mm256_shuffle_ps(row_scale, row_scale, 0)), mn[0]);
                mn[1] = _mm256_fmadd_ps(_mm256_cvtepi32_ps(m[1]), _mm256_mul_ps(col_dmin, _mm256_shuffle_ps(row_scale, row_scale, 85)), mn[1]);
                mn[2] = _mm256_fmadd_ps(_mm256_cvtepi32_ps(m[2]), _mm256_mul_ps(col_dmin, _mm256_shuffle_ps(row_scale, row_scale, 170)), mn[2]);
                mn[3] = _mm256_fmadd_ps(_mm256_cvtepi32_ps(m[3]), _mm256_mul_ps(col_dmin, _mm256_shuffle_ps(row_scale, row_scale, 255)), mn[3]);
            }
            for (int r = 0; r < 4; r++)
                _mm256_storeu_ps(dst + (long)(yy * 4 + r) * ldc + xx * 8,
                                 _mm256_sub_ps(_mm256_permutevar8x32_ps(acc[r], col_perm), mn[r]));
        }
    }
}

/* GemmQ4K.GemmAvx2 (GemmQ4K.Avx2.cs:25-35): 128 KiB column tiles. */
static void gemm_avx2(int n, float* dst, int ldc, const uint8_t* weights, const uint8_t* acts,
                      int rows, int cols, const uint8_t* meta)
{
    int nb = n / OQ_QK;
    int tile_groups = (128 * 1024) / (nb * OQ_Q4KX8_BYTES);
    if (tile_groups < 1) tile_groups = 1;
    int groups = cols / 8;
    for (int g0 = 0; g0 < groups; g0 += tile_groups) {
        int g1 = g0 + tile_groups < groups ? g0 + tile_groups : groups;
        gemm_avx2_tile(n, dst + g0 * 8, ldc, weights + (long)g0 * nb * OQ_Q4KX8_BYTES, acts, rows,
                       (g1 - g0) * 8, meta + (long)g0 * nb * OQ_Q4KX8_META_BYTES);
    }
}

/* ---- Thread pool (CpuThreadPool.For / Barrier, CpuThreadPool.cs:46-131) --
 * Persistent workers; For(count) runs body(worker, workers) on
 * workers = min(threads, count) pool threads while the caller waits;
 * count <= 1 or a single-thread pool runs inline.  Idle workers spin briefly,
 * then sleep on a condition variable (the reference parks on an event). */

typedef void (*oq_body)(void* arg, int worker, int workers);

typedef struct {
    int nthreads;
    pthread_t* threads;
    pthread_mutex_t mu;
    pthread_cond_t cv;
    atomic_int gen;
    atomic_int remaining;
    atomic_int barrier_count;
    atomic_int barrier_gen;
    int workers;
    int stop;
    oq_body fn;
    void* arg;
} oq_pool;

static oq_pool* g_pool;

static void* pool_worker(void* p)
{
    long index = (long)p;
    int seen = 0;
    for (;;) {
        int spins = 0;
        while (atomic_load_explicit(&g_pool->gen, memory_order_acquire) == seen) {
            if (++spins < 20000) {
                _mm_pause();
                continue;
            }
            pthread_mutex_lock(&g_pool->mu);
            while (atomic_load(&g_pool->gen) == seen)
                pthread_cond_wait(&g_pool->cv, &g_pool->mu);
            pthread_mutex_unlock(&g_pool->mu);
        }
        seen = atomic_load(&g_pool->gen);
        if (g_pool->stop)
            return NULL;
        if (index < g_pool->workers) {
            g_pool->fn(g_pool->arg, (int)index, g_pool->workers);
            atomic_fetch_sub_explicit(&g_pool->remaining, 1, memory_order_release);
        }
    }
}

static void pool_shutdown(void)
{
    if (!g_pool)
        return;
    pthread_mutex_lock(&g_pool->mu);
    g_pool->stop = 1;
    atomic_fetch_add(&g_pool->gen, 1);
    pthread_cond_broadcast(&g_pool->cv);
    pthread_mutex_unlock(&g_pool->mu);
    for (int i = 0; i < g_pool->nthreads; i++)
        pthread_join(g_pool->threads[i], NULL);
    free(g_pool->threads);
    free(g_pool);
    g_pool = NULL;
}

static void pool_ensure(int threads)
{
    if (threads < 1) threads = 1;
    if (g_pool && g_pool->nthreads == threads)
        return;
    pool_shutdown();
    g_pool = (oq_pool*)calloc(1, sizeof(oq_pool));
    g_pool->nthreads = threads;
    pthread_mutex_init(&g_pool->mu, NULL);
    pthread_cond_init(&g_pool->cv, NULL);
    g_pool->threads = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
    for (long i = 0; i < threads; i++)
        pthread_create(&g_pool->threads[i], NULL, pool_worker, (void*)i);
}

static void pool_for(int threads, int count, oq_body fn, void* arg)
{
    if (count <= 1 || threads <= 1) {
        fn(arg, 0, 1);
        return;
    }
    pool_ensure(threads);
    int workers = threads < count ? threads : count;
    g_pool->fn = fn;
    g_pool->arg = arg;
    g_pool->workers = workers;
    atomic_store(&g_pool->remaining, workers);
    atomic_store(&g_pool->barrier_count, 0);
    pthread_mutex_lock(&g_pool->mu);
    atomic_fetch_add_explicit(&g_pool->gen, 1, memory_order_release);
    pthread_cond_broadcast(&g_pool->cv);
    pthread_mutex_unlock(&g_pool->mu);
    while (atomic_load_explicit(&g_pool->remaining, memory_order_acquire) > 0)
        _mm_pause();
}

static void pool_barrier(int workers)
{
    int n = workers;
    if (n <= 1 || !g_pool)
        return;
    int gen = atomic_load(&g_pool->barrier_gen);
    if (atomic_fetch_add(&g_pool->barrier_count, 1) + 1 == n) {
        atomic_store(&g_pool->barrier_count, 0);
        atomic_fetch_add(&g_pool->barrier_gen, 1);
        return;
    }
    while (atomic_load(&g_pool->barrier_gen) == gen)
        _mm_pause();
}

/* ---- Prepared weights and dispatch ------------------------------------ */

struct oq_weight {
    int type, nIn, nOut, nb;
    const uint8_t* rows;
    uint8_t* packed; /* Q4_K: BlockQ4Kx8 panel (nOut/8 groups) */
    uint8_t* meta;   /* Q4_K: BlockQ4Kx8Meta sidecar */
};

oq_weight* oq_weight_prepare(int type, const void* blocks, int nIn, int nOut)
{
    if (oq_block_bytes(type) == 0 || nIn % OQ_QK != 0 || nOut <= 0)
        return NULL;
    oq_weight* w = (oq_weight*)calloc(1, sizeof(oq_weight));
    w->type = type;
    w->nIn = nIn;
    w->nOut = nOut;
    w->nb = nIn / OQ_QK;
    w->rows = (const uint8_t*)blocks;
    if (type == OQ_Q4_K && nOut >= 8) {
        long groups = nOut / 8;
        w->packed = (uint8_t*)aligned_alloc(64, (size_t)(groups * w->nb * OQ_Q4KX8_BYTES + 64));
        w->meta = (uint8_t*)aligned_alloc(64, (size_t)(groups * w->nb * OQ_Q4KX8_META_BYTES + 64));
        oq_repack_q4kx8(blocks, w->packed, nIn, (int)(groups * 8));
        oq_build_meta_q4kx8(blocks, w->meta, nIn, (int)(groups * 8));
    }
    return w;
}

void oq_weight_release(oq_weight* w)
{
    if (!w)
        return;
    free(w->packed);
    free(w->meta);
    free(w);
}

typedef struct {
    const oq_weight* w;
    const uint8_t* q8;
    float* y;
} gemv_job;

/* GemvPrequant bodies (MulMatQ4K.cs:28-43, Q5K.cs:97-112, Q6K.cs:415-430):
 * rows [nOut*w/W, nOut*(w+1)/W). */
static void gemv_body(void* p, int worker, int workers)
{
    gemv_job* j = (gemv_job*)p;
    const oq_weight* w = j->w;
    long row_bytes = (long)w->nb * oq_block_bytes(w->type);
    int begin = (int)((long)w->nOut * worker / workers);
    int end = (int)((long)w->nOut * (worker + 1) / workers);
    for (int row = begin; row < end; row++)
        j->y[row] = oq_dot_avx2(w->type, w->rows + row * row_bytes, j->q8, w->nIn);
}

static void gemv_prequant(const oq_weight* w, const uint8_t* q8, float* y, int threads)
{
    gemv_job j = {w, q8, y};
    pool_for(threads, w->nOut, gemv_body, &j);
}

typedef struct {
    const oq_weight* w;
    const float* input;
    uint8_t* q8;
    float* dst;
    int tokens;
} q4gemm_job;

/* MulMatQ4K.QuantizeAndGemmPrequant body (MulMatQ4K.cs:163-186). */
static void q4gemm_body(void* p, int worker, int workers)
{
    q4gemm_job* j = (q4gemm_job*)p;
    const oq_weight* w = j->w;
    int nb = w->nb;
    int quant_groups = j->tokens / 4;
    int gemm_groups = (w->nOut & ~7) / 8;
    int q0 = (int)((long)quant_groups * worker / workers);
    int q1 = (int)((long)quant_groups * (worker + 1) / workers);
    for (int g = q0; g < q1; g++)
        oq_quantize_q8kx4(j->input + (long)g * 4 * w->nIn, j->q8 + (long)g * nb * OQ_Q8KX4_BYTES, w->nIn);
    pool_barrier(workers);
    if (gemm_groups == 0)
        return;
    int g0 = (int)((long)gemm_groups * worker / workers);
    int g1 = (int)((long)gemm_groups * (worker + 1) / workers);
    if (g0 >= g1)
        return;
    gemm_avx2(w->nIn, j->dst + g0 * 8, w->nOut, w->packed + (long)g0 * nb * OQ_Q4KX8_BYTES, j->q8,
              j->tokens, (g1 - g0) * 8, w->meta + (long)g0 * nb * OQ_Q4KX8_META_BYTES);
}

/* MulMatQ4K.Gemm, tokens > 1 (MulMatQ4K.cs:45-127). */
static void q4k_gemm(const oq_weight* w, const float* input, float* output, int tokens, int threads)
{
    int nIn = w->nIn, nOut = w->nOut, nb = w->nb;
    int padded = (tokens + 3) & ~3;
    int packed_cols = nOut & ~7;
    int aligned = padded == tokens;
    uint8_t* q8 = (uint8_t*)aligned_alloc(64, (size_t)(padded / 4) * nb * OQ_Q8KX4_BYTES + 64);
    const float* src = input;
    float* dst = output;
    float* staging = NULL;
    float* scratch_out = NULL;
    if (!aligned) {
        staging = (float*)calloc((size_t)padded * nIn, sizeof(float));
        scratch_out = (float*)calloc((size_t)padded * nOut, sizeof(float));
        memcpy(staging, input, (size_t)tokens * nIn * sizeof(float));
        src = staging;
        dst = scratch_out;
    }
    {
        q4gemm_job j = {w, src, q8, dst, padded};
        int quant_groups = padded / 4, gemm_groups = packed_cols / 8;
        int jobs = gemm_groups > 1 ? gemm_groups : 1;
        if (quant_groups > jobs)
            jobs = quant_groups;
        pool_for(threads, jobs, q4gemm_body, &j);
    }
    if (packed_cols < nOut) {
        uint8_t* q8row = (uint8_t*)aligned_alloc(64, (size_t)nb * OQ_Q8K_BYTES + 64);
        long row_bytes = (long)nb * OQ_Q4K_BYTES;
        for (int t = 0; t < tokens; t++) {
            oq_quantize_q8k_avx2(input + (long)t * nIn, q8row, nIn);
            for (int row = packed_cols; row < nOut; row++)
                dst[(long)t * nOut + row] = dot_q4k_avx2(w->rows + row * row_bytes, q8row, nIn);
        }
        free(q8row);
    }
    if (!aligned)
        memcpy(output, dst, (size_t)tokens * nOut * sizeof(float));
    free(staging);
    free(scratch_out);
    free(q8);
}

typedef struct {
    const oq_weight* w;
    const float* input;
    uint8_t* q8;
    float* output;
    int tokens;
} q6gemm_job;

/* Q6K.Gemm pooled body (Q6K.cs:337-345) + GemmFromQ8Range (Q6K.cs:380-413). */
static void q6gemm_body(void* p, int worker, int workers)
{
    q6gemm_job* j = (q6gemm_job*)p;
    const oq_weight* w = j->w;
    int nb = w->nb, nIn = w->nIn, nOut = w->nOut, tokens = j->tokens;
    int t0 = (int)((long)tokens * worker / workers), t1 = (int)((long)tokens * (worker + 1) / workers);
    for (int t = t0; t < t1; t++)
        oq_quantize_q8k_avx2(j->input + (long)t * nIn, j->q8 + (long)t * nb * OQ_Q8K_BYTES, nIn);
    pool_barrier(workers);
    int begin = (int)((long)nOut * worker / workers), end = (int)((long)nOut * (worker + 1) / workers);
    long row_bytes = (long)nb * OQ_Q6K_BYTES;
    long q8_row = (long)nb * OQ_Q8K_BYTES;
    int t = 0;
    float tmp[4];
    for (; t + 3 < tokens; t += 4) {
        for (int row = begin; row < end; row++) {
            oq_dot_q6k_avx2x4(w->rows + row * row_bytes, j->q8 + t * q8_row, j->q8 + (t + 1) * q8_row,
                              j->q8 + (t + 2) * q8_row, j->q8 + (t + 3) * q8_row, nIn, tmp);
            for (int u = 0; u < 4; u++)
                j->output[(long)(t + u) * nOut + row] = tmp[u];
        }
    }
    for (; t < tokens; t++)
        for (int row = begin; row < end; row++)
            j->output[(long)t * nOut + row] = dot_q6k_avx2(w->rows + row * row_bytes, j->q8 + t * q8_row, nIn);
}

int oq_matmul(const oq_weight* w, const float* x, float* y, int tokens, int threads)
{
    if (!w || tokens <= 0)
        return -1;
    int nb = w->nb;
    if (w->type == OQ_Q6_K && tokens > 1) {
        uint8_t* q8 = (uint8_t*)aligned_alloc(64, (size_t)tokens * nb * OQ_Q8K_BYTES + 64);
        q6gemm_job j = {w, x, q8, y, tokens};
        int count = tokens > w->nOut ? tokens : w->nOut;
        pool_for(threads, count, q6gemm_body, &j);
        free(q8);
        return 0;
    }
    if (w->type == OQ_Q4_K && tokens > 1) {
        q4k_gemm(w, x, y, tokens, threads);
        return 0;
    }
    /* Gemv (Q4_K/Q6_K tokens==1) and Q5K.Gemm's per-token Gemv loop. */
    uint8_t* q8 = (uint8_t*)aligned_alloc(64, (size_t)nb * OQ_Q8K_BYTES + 64);
    for (int t = 0; t < tokens; t++) {
        oq_quantize_q8k_avx2(x + (long)t * w->nIn, q8, w->nIn);
        gemv_prequant(w, q8, y + (long)t * w->nOut, threads);
    }
    free(q8);
    return 0;
}

int oq_matmul_q8k(const oq_weight* w, const void* q8k, float* y, int tokens, int threads)
{
    if (!w || tokens <= 0)
        return -1;
    const uint8_t* q8 = (const uint8_t*)q8k;
    for (int t = 0; t < tokens; t++)
        gemv_prequant(w, q8 + (long)t * w->nb * OQ_Q8K_BYTES, y + (long)t * w->nOut, threads);
    return 0;
}

int oq_matmul_semantic(const oq_weight* w, const float* x, float* y, int tokens)
{
    if (!w || tokens <= 0)
        return -1;
    int nb = w->nb, nIn = w->nIn, nOut = w->nOut;
    long row_bytes = (long)nb * oq_block_bytes(w->type);
    uint8_t* q8 = (uint8_t*)aligned_alloc(64, (size_t)tokens * nb * OQ_Q8K_BYTES + 64);
    for (int t = 0; t < tokens; t++)
        oq_quantize_q8k_scalar(x + (long)t * nIn, q8 + (long)t * nb * OQ_Q8K_BYTES, nIn);
    if (w->type == OQ_Q4_K && tokens > 1) {
        /* Panel GEMM semantics on the padded token count; the nOut%8 tail
         * uses the row dot (MulMatQ4K.cs:98-116). */
        int padded = (tokens + 3) & ~3, cols = nOut & ~7;
        uint8_t* q8p = (uint8_t*)calloc((size_t)padded * nb, OQ_Q8K_BYTES);
        memcpy(q8p, q8, (size_t)tokens * nb * OQ_Q8K_BYTES);
        float* tmp = (float*)calloc((size_t)padded * nOut, sizeof(float));
        if (cols > 0)
            oq_gemm_q4k_semantic(w->rows, q8p, tmp, nOut, nIn, padded, cols);
        for (int t = 0; t < tokens; t++) {
            for (int row = cols; row < nOut; row++)
                tmp[(long)t * nOut + row] = oq_dot_scalar(OQ_Q4_K, w->rows + row * row_bytes, q8 + (long)t * nb * OQ_Q8K_BYTES, nIn);
            memcpy(y + (long)t * nOut, tmp + (long)t * nOut, (size_t)nOut * sizeof(float));
        }
        free(tmp);
        free(q8p);
    } else {
        for (int t = 0; t < tokens; t++)
            for (int row = 0; row < nOut; row++)
                y[(long)t * nOut + row] = oq_dot_scalar(w->type, w->rows + row * row_bytes, q8 + (long)t * nb * OQ_Q8K_BYTES, nIn);
    }
    free(q8);
    return 0;
}
