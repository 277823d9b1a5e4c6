// Checker: the library's restated expf (cosxamix_b200/csrc/expf_glibc.h, host
// path) against the host libm expf over every float whose bit pattern is
// congruent to `phase` modulo `stride`. Prints the mismatch count.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "../cosxamix_b200/csrc/expf_glibc.h"

int main(int argc, char **argv) {
    unsigned long stride = argc > 1 ? strtoul(argv[1], nullptr, 10) : 1;
    unsigned long phase = argc > 2 ? strtoul(argv[2], nullptr, 10) : 0;
    unsigned long n = 0, bad = 0;
    for (unsigned long u = phase; u <= 0xFFFFFFFFul; u += stride) {
        uint32_t b = (uint32_t)u;
        float x;
        memcpy(&x, &b, 4);
        float a = expf(x), c = cxm::expf_glibc(x);
        n++;
        if (memcmp(&a, &c, 4) != 0 && !(std::isnan(a) && std::isnan(c))) bad++;
    }
    printf("%lu %lu\n", n, bad);
    return 0;
}
