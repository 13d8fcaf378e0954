/* expf_table.c -- build step of libqwen_moe_b200.so.
 *
 * The reference's CPU expert computes SiLU with the C library's expf
 * (src/cpu_expert.cpp:248-259).  The device computes exp in double precision
 * and rounds once (correctly rounded for all practical purposes); the C
 * library's expf is not correctly rounded on every input.  This program runs
 * the C library's expf on every float input whose result is finite and
 * nonzero -- x in [-104, 89] -- and writes the inputs where it differs from
 * the once-rounded double exp, as little-endian uint32 pairs
 * (x bits, expf(x) bits) in ascending order of x bits, to the file named by
 * argv[1].  The library loads the pairs into a device hash table, so the
 * device's exp equals this C library's expf bit for bit.
 *
 *   cc -O2 expf_table.c -o expf_table -lm && ./expf_table out.bin
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

static int emit(FILE *f, uint32_t xb) {
    float x, y, z;
    memcpy(&x, &xb, 4);
    y = expf(x);
    z = (float)exp((double)x);
    if (y == z || (y != y && z != z)) return 0;
    uint32_t yb;
    memcpy(&yb, &y, 4);
    const uint32_t pair[2] = {xb, yb};
    return fwrite(pair, 4, 2, f) == 2 ? 1 : -1;
}

int main(int argc, char **argv) {
    if (argc != 2) {
        fprintf(stderr, "usage: %s out.bin\n", argv[0]);
        return 2;
    }
    FILE *f = fopen(argv[1], "wb");
    if (!f) return 1;
    long n = 0;
    /* ascending bit patterns: +0 .. 89.0, then -0 .. -104.0 */
    for (uint32_t u = 0; u <= 0x42b20000u; ++u) {
        const int r = emit(f, u);
        if (r < 0) return 1;
        n += r;
    }
    for (uint32_t u = 0x80000000u; u <= 0xc2d00000u; ++u) {
        const int r = emit(f, u);
        if (r < 0) return 1;
        n += r;
    }
    if (fclose(f) != 0) return 1;
    printf("%ld corrections\n", n);
    return 0;
}
