/* Exhaustive host check of the encode arithmetic used by the sm_100a kernels.
 *
 * Compiles the product's glint_codec.cuh and its generated lookup table on the
 * host and compares them with the CPU oracle (oracle/glint_oracle.c, the
 * restatement of reference cuda/glint_encode.cu:67-102):
 *
 *   codes   every f32 bit pattern v with |v| <= 1, and every quiet NaN:
 *           table lookup == oracle scan (orc_code).  Signalling NaNs are left
 *           out: the quotient v is always the result of arithmetic, which never
 *           returns a signalling NaN, and the host's fmaxf treats them unlike
 *           the GPU's max instruction.
 *   bf16div every BF16 pair (w, s) with 0 < s finite, |w| <= s:
 *           code(Markstein quotient) == code(IEEE w / s), and the quotient bits
 *           agree whenever |w / s| >= 2^-20
 *   f32div  random f32 pairs (w, s), |w| <= s, s in the Markstein range, plus
 *           pairs with w and s within a few ulps of each other
 *
 * Prints "OK <mode> <count>" or the first mismatches and exits 1.
 * Build: g++ -O2 -fopenmp -std=c++17 -I<lut dir> check_codes.cpp -L<oracle> -lglint_oracle
 */
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <omp.h>

#include "../../glint_b200/csrc/glint_codec.cuh"
#include "glint_lut.inc"

extern "C" int orc_code(float v);

static inline uint32_t lookup(float v)
{
    uint32_t c = glint::cell_of(v);
    glint::CellEntry e{glint::u2f(GLINT_LUT_ENTRIES[c][0]), GLINT_LUT_ENTRIES[c][1]};
    return glint::code_from_entry(v, e);
}

static int mode_codes()
{
    std::atomic<long long> bad{0}, checked{0};
    const uint32_t one = 0x3F800000u;
#pragma omp parallel for schedule(dynamic, 1)
    for (int chunk = 0; chunk < 4096; ++chunk) {
        long long lbad = 0, lchk = 0;
        uint32_t lo = (uint32_t)chunk << 20;
        for (uint32_t i = 0; i < (1u << 20); ++i) {
            uint32_t u = lo + i;
            uint32_t mag = u & 0x7FFFFFFFu;
            bool qnan = mag >= 0x7FC00000u;
            if (mag > one && !qnan)
                continue;
            float v = glint::u2f(u);
            ++lchk;
            if ((int)lookup(v) != orc_code(v)) {
                if (lbad < 4)
                    printf("MISMATCH codes v=%a bits=%08x lookup=%u oracle=%d\n", v, u, lookup(v), orc_code(v));
                ++lbad;
            }
        }
        bad += lbad;
        checked += lchk;
    }
    if (bad) {
        printf("FAIL codes mismatches=%lld of %lld\n", (long long)bad, (long long)checked);
        return 1;
    }
    printf("OK codes %lld\n", (long long)checked);
    return 0;
}

/* the kernel's quotient for one weight: IEEE outside the Markstein range */
static inline float kernel_quotient(float w, float s)
{
    if (s == 0.0f)
        return 0.0f;
    if (s >= glint::kMarksteinLo && s <= glint::kMarksteinHi) {
        float y = glint::div_rn(1.0f, s);
        return glint::quotient_markstein(w, s, y);
    }
    return glint::div_rn(w, s);
}

static bool same(float w, float s, long long &bits_checked)
{
    float q = kernel_quotient(w, s);
    float r = (s == 0.0f) ? 0.0f : glint::div_rn(w, s);
    if (lookup(q) != lookup(r))
        return false;
    if (!std::isnan(r) && fabsf(r) >= 9.5367431640625e-07f) { /* 2^-20 */
        ++bits_checked;
        return glint::f2u(q) == glint::f2u(r);
    }
    return true;
}

static int mode_bf16div()
{
    std::atomic<long long> bad{0}, checked{0}, bits{0};
#pragma omp parallel for schedule(dynamic, 16)
    for (int sb = 1; sb < 0x7F80; ++sb) {
        float s = glint::bf16_bits_to_f32((uint32_t)sb);
        long long lbad = 0, lchk = 0, lbits = 0;
        for (uint32_t wb = 0; wb < 0x10000u; ++wb) {
            if ((wb & 0x7FFFu) > (uint32_t)sb)
                continue; /* |w| > s cannot occur in a block whose absmax is s */
            float w = glint::bf16_bits_to_f32(wb);
            ++lchk;
            if (!same(w, s, lbits)) {
                if (lbad < 4)
                    printf("MISMATCH bf16div w=%a s=%a q=%a ieee=%a\n", w, s, kernel_quotient(w, s), glint::div_rn(w, s));
                ++lbad;
            }
        }
        bad += lbad;
        checked += lchk;
        bits += lbits;
    }
    if (bad) {
        printf("FAIL bf16div mismatches=%lld of %lld\n", (long long)bad, (long long)checked);
        return 1;
    }
    printf("OK bf16div %lld (quotient bits compared on %lld)\n", (long long)checked, (long long)bits);
    return 0;
}

static int mode_f32div(long long samples)
{
    std::atomic<long long> bad{0}, bits{0};
#pragma omp parallel
    {
        std::mt19937_64 rng(12345u + 977u * (unsigned)omp_get_thread_num());
        long long lbad = 0, lbits = 0;
#pragma omp for schedule(static)
        for (long long i = 0; i < samples; ++i) {
            /* s: any f32 in [2^-60, 2^60]; w: |w| <= s, either random or a few ulps below s */
            uint32_t sexp = 67 + (uint32_t)(rng() % 120); /* biased exponent 67..186 */
            uint32_t sbits = (sexp << 23) | (uint32_t)(rng() & 0x7FFFFFu);
            float s = glint::u2f(sbits);
            float w;
            uint64_t r = rng();
            if ((r & 3) == 0) {
                w = glint::u2f(sbits - (uint32_t)((r >> 2) % 64));
            } else {
                uint32_t wexp = (uint32_t)((r >> 8) % (sexp + 1));
                uint32_t wbits = (wexp << 23) | (uint32_t)((r >> 16) & 0x7FFFFFu);
                w = glint::u2f(wbits);
                if (fabsf(w) > s)
                    w = s;
            }
            if (r & (1ull << 40))
                w = -w;
            if (!same(w, s, lbits)) {
                if (lbad < 4)
                    printf("MISMATCH f32div w=%a s=%a q=%a ieee=%a\n", w, s, kernel_quotient(w, s), glint::div_rn(w, s));
                ++lbad;
            }
        }
        bad += lbad;
        bits += lbits;
    }
    if (bad) {
        printf("FAIL f32div mismatches=%lld of %lld\n", (long long)bad, samples);
        return 1;
    }
    printf("OK f32div %lld (quotient bits compared on %lld)\n", samples, (long long)bits);
    return 0;
}

int main(int argc, char **argv)
{
    if (argc < 2) {
        fprintf(stderr, "usage: check_codes codes|bf16div|f32div [samples]\n");
        return 2;
    }
    if (!strcmp(argv[1], "codes"))
        return mode_codes();
    if (!strcmp(argv[1], "bf16div"))
        return mode_bf16div();
    if (!strcmp(argv[1], "f32div"))
        return mode_f32div(argc > 2 ? atoll(argv[2]) : (1ll << 26));
    fprintf(stderr, "unknown mode %s\n", argv[1]);
    return 2;
}
