/*
 * Oracle SIMD ports (test infrastructure only; see oracle.h).
 *
 * oq_gemv_q4_avx2   restates simd.rs:76-153  (gemv_q4_avx2)
 * oq_gemv_q4_avx512 restates simd.rs:203-269 (gemv_q4_avx512)
 *
 * Both keep the scalar kernel's k-major order and produce the same bits
 * (the reference asserts this for AVX2 in gemv.rs:735-773; the same
 * assertion is restated for both ports in tests/).
 */
#include "oracle.h"

#include <immintrin.h>
#include <string.h>

int oq_has_avx2(void) { return __builtin_cpu_supports("avx2"); }
int oq_has_avx512(void) { return __builtin_cpu_supports("avx512f"); }

__attribute__((target("avx2"))) void oq_gemv_q4_avx2(const float *input, const uint8_t *packed,
                                                       const uint16_t *scales, int64_t n,
                                                       int64_t k_start, int64_t k_end,
                                                       float *output) {
    int64_t gpr = n / 32, ppr = gpr * 16;
    memset(output, 0, sizeof(float) * (size_t)n);
    const __m256i nibble_mask = _mm256_set1_epi32(0x0F);
    const __m256 eight = _mm256_set1_ps(8.0f);
    for (int64_t ki = k_start; ki < k_end; ki++) {
        float val = input[ki];
        if (val == 0.0f) continue;
        int64_t sb = ki * gpr, pb = ki * ppr;
        for (int64_t g = 0; g < gpr; g++) {
            float s = oq_f16_to_f32(scales[sb + g]) * val;
            if (s == 0.0f) continue;
            __m256 s_vec = _mm256_set1_ps(s);
            __m128i bytes = _mm_loadu_si128((const __m128i *)(packed + pb + g * 16));
            for (int h = 0; h < 2; h++) {
                __m128i half = h == 0 ? bytes : _mm_srli_si128(bytes, 8);
                __m256i v8 = _mm256_cvtepu8_epi32(half);
                __m256i lo = _mm256_and_si256(v8, nibble_mask);
                __m256i hi = _mm256_srli_epi32(v8, 4);
                __m256 lo_v = _mm256_mul_ps(_mm256_sub_ps(_mm256_cvtepi32_ps(lo), eight), s_vec);
                __m256 hi_v = _mm256_mul_ps(_mm256_sub_ps(_mm256_cvtepi32_ps(hi), eight), s_vec);
                __m256 a = _mm256_unpacklo_ps(lo_v, hi_v);
                __m256 b = _mm256_unpackhi_ps(lo_v, hi_v);
                __m256 first = _mm256_permute2f128_ps(a, b, 0x20);
                __m256 second = _mm256_permute2f128_ps(a, b, 0x31);
                int64_t oo = g * 32 + h * 16;
                _mm256_storeu_ps(output + oo, _mm256_add_ps(_mm256_loadu_ps(output + oo), first));
                _mm256_storeu_ps(output + oo + 8,
                                 _mm256_add_ps(_mm256_loadu_ps(output + oo + 8), second));
            }
        }
    }
}

static const float Q4_FACTORS[16] = {-8, -7, -6, -5, -4, -3, -2, -1, 0, 1, 2, 3, 4, 5, 6, 7};
static const int32_t INTERLEAVE_FIRST[16] = {0, 16, 1, 17, 2, 18, 3, 19,
                                             4, 20, 5, 21, 6, 22, 7, 23};
static const int32_t INTERLEAVE_SECOND[16] = {8, 24, 9, 25, 10, 26, 11, 27,
                                              12, 28, 13, 29, 14, 30, 15, 31};

__attribute__((target("avx512f"))) void oq_gemv_q4_avx512(const float *input,
                                                            const uint8_t *packed,
                                                            const uint16_t *scales, int64_t n,
                                                            int64_t k_start, int64_t k_end,
                                                            float *output) {
    int64_t gpr = n / 32, ppr = gpr * 16;
    memset(output, 0, sizeof(float) * (size_t)n);
    const __m512 factors = _mm512_loadu_ps(Q4_FACTORS);
    const __m512i il_lo = _mm512_loadu_si512((const void *)INTERLEAVE_FIRST);
    const __m512i il_hi = _mm512_loadu_si512((const void *)INTERLEAVE_SECOND);
    const __m512i nibble_mask = _mm512_set1_epi32(0x0F);
    for (int64_t ki = k_start; ki < k_end; ki++) {
        float val = input[ki];
        if (val == 0.0f) continue;
        int64_t sb = ki * gpr, pb = ki * ppr;
        for (int64_t g = 0; g < gpr; g++) {
            float s = oq_f16_to_f32(scales[sb + g]) * val;
            if (s == 0.0f) continue;
            __m512 lut = _mm512_mul_ps(factors, _mm512_set1_ps(s));
            __m128i bytes = _mm_loadu_si128((const __m128i *)(packed + pb + g * 16));
            __m512i b32 = _mm512_cvtepu8_epi32(bytes);
            __m512i lo = _mm512_and_epi32(b32, nibble_mask);
            __m512i hi = _mm512_srli_epi32(b32, 4);
            __m512 lo_v = _mm512_permutexvar_ps(lo, lut);
            __m512 hi_v = _mm512_permutexvar_ps(hi, lut);
            __m512 first = _mm512_permutex2var_ps(lo_v, il_lo, hi_v);
            __m512 second = _mm512_permutex2var_ps(lo_v, il_hi, hi_v);
            int64_t oo = g * 32;
            _mm512_storeu_ps(output + oo, _mm512_add_ps(_mm512_loadu_ps(output + oo), first));
            _mm512_storeu_ps(output + oo + 16,
                             _mm512_add_ps(_mm512_loadu_ps(output + oo + 16), second));
        }
    }
}
