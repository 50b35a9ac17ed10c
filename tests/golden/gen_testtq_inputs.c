/*
 * gen_testtq_inputs.c — regenerates the input vectors of LeanKV's own C tests
 * so their printed results can be pinned as known answers.
 *
 * Restates the deterministic generator of src/test-tq.c:51-64 (xorshift32 and
 * a Box-Muller normal from two 16-bit uniforms) and the data construction of
 * tests T2 (:172-210), T3 (:214-242), T6 (:327-391) and T9 (:501-595).
 * Built with the reference's flags (-O2 -std=c11) so libm's logf/cosf/sqrtf
 * give the same floats as the reference test binary.
 *
 * Output: raw float32 little-endian, concatenated in this order:
 *   t2[1024] t3[1024] t6[256] t9_k[128*64] t9_q[64]
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>

static uint32_t next_u32(uint32_t *s) {
    uint32_t v = *s;
    v ^= v << 13;
    v ^= v >> 17;
    v ^= v << 5;
    *s = v;
    return v;
}

static float normal(uint32_t *s) {
    float a = (float)(next_u32(s) & 0xFFFF) / 65535.0f;
    float b = (float)(next_u32(s) & 0xFFFF) / 65535.0f;
    if (a < 1e-10f) a = 1e-10f;
    return sqrtf(-2.0f * logf(a)) * cosf(6.2831853f * b);
}

static void put(const float *v, int n) { fwrite(v, sizeof(float), (size_t)n, stdout); }

int main(void) {
    static float t2[1024], t3[1024], t6[256], k9[128 * 64], q9[64];
    uint32_t s;

    s = 12345;                                   /* T2: sigma 0.125 */
    for (int i = 0; i < 1024; ++i) t2[i] = normal(&s) * 0.125f;
    s = 54321;                                   /* T3 */
    for (int i = 0; i < 1024; ++i) t3[i] = normal(&s) * 0.125f;

    s = 777;                                     /* T6: 4 heads of 64, one outlier each */
    for (int i = 0; i < 256; ++i) t6[i] = normal(&s) * 0.1f;
    for (int h = 0; h < 4; ++h) t6[h * 64 + (h * 17 + 3) % 64] = normal(&s) * 2.0f;

    s = 555;                                     /* T9: K [128][64], Q [64], K outliers x20 */
    for (int i = 0; i < 128 * 64; ++i) k9[i] = normal(&s) * 0.1f;
    for (int i = 0; i < 64; ++i) q9[i] = normal(&s) * 0.1f;
    for (int t = 0; t < 128; ++t) k9[t * 64 + (t * 13 + 7) % 64] *= 20.0f;

    put(t2, 1024);
    put(t3, 1024);
    put(t6, 256);
    put(k9, 128 * 64);
    put(q9, 64);
    return 0;
}
