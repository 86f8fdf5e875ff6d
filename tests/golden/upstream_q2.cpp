// Golden-vector program (run by tests/golden/make_golden.py, in the container that holds the
// reference tree). Includes the reference's upstream Q2_0 contract header where it lies
// (vendor/strata/include/strata/artifact/dequant.hpp:33-78) and writes, as raw little-endian
// floats: fp16_to_fp32 of all 65,536 halves, then dequantize_q2_0 of the 256 closed-form
// blocks that the reference's own upstream check builds (scripts/test-upstream.mjs:21).
#include "strata/artifact/dequant.hpp"

#include <cstdio>

int main(int argc, char **argv) {
    if (argc != 2) return 2;
    FILE *f = std::fopen(argv[1], "wb");
    if (!f) return 3;
    for (unsigned h = 0; h < 65536; ++h) {
        float v = strata::fp16_to_fp32((uint16_t)h);
        std::fwrite(&v, 4, 1, f);
    }
    for (int b = 0; b < 256; ++b) {
        unsigned char block[18];
        unsigned h = ((b % 16) + 8) * 1024 + (b * 7) % 1024 + (b % 2 ? 32768 : 0);
        block[0] = h & 255;
        block[1] = h >> 8;
        for (int i = 0; i < 16; ++i) block[2 + i] = (unsigned char)((i * 19 + b * 73) & 255);
        float values[64];
        strata::dequantize_q2_0(block, values);
        std::fwrite(values, 4, 64, f);
    }
    return std::fclose(f) == 0 ? 0 : 4;
}
