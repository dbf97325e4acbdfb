// 2:4 weight compression for the sparse projections (layout: gemm_sp.cuh). Host code: runs once per weight at
// engine bring-up (or through xtb_sparse24_compress). The selection of which two of every four weights to keep
// is the converter's (prune24.py:44-56, restated in oracle/ as or_prune24); this file only packs weights that
// are already 2:4 into the form tcgen05.mma.sp reads.
#include <stdio.h>
#include <string.h>

#include "ops.h"

namespace xtb {

static inline int round128(int x) { return (x + 127) & ~127; }
static inline bool nonzero(uint8_t c) { return (c & 0x7F) != 0; }  // E4M3 0x00 and 0x80 are zeros

int sparse24_check(const uint8_t *w, int n, int k)
{
    if (!w || n <= 0 || k <= 0 || (k & 3)) return 0;
    for (size_t r = 0; r < (size_t)n; r++) {
        const uint8_t *src = w + r * k;
        for (int g = 0; g < k; g += 4)
            if (nonzero(src[g]) + nonzero(src[g + 1]) + nonzero(src[g + 2]) + nonzero(src[g + 3]) > 2) return 0;
    }
    return 1;
}

size_t sparse24_bytes(int n, int k, size_t *meta_off)
{
    const size_t np = round128(n), kp = round128(k);
    if (meta_off) *meta_off = np * kp / 2;
    return np * kp / 2 + np * kp / 8;
}

int sparse24_compress(const uint8_t *w, int n, int k, uint8_t *vals, uint8_t *meta)
{
    if (!sparse24_check(w, n, k)) {
        fprintf(stderr, "eva: weight [%d][%d] is not 2:4 sparse along k (or k is not a multiple of 4)\n", n, k);
        return -1;
    }
    const size_t np = round128(n), vl = round128(k) / 2, ml = round128(k) / 8;
    memset(vals, 0, np * vl);
    memset(meta, 0x44, np * ml);  // padding groups (rows past n, k past the end): indices 0 and 1, zero values
    for (size_t r = 0; r < (size_t)n; r++) {
        const uint8_t *src = w + r * k;
        uint8_t *v = vals + r * vl, *m = meta + r * ml;
        for (int g = 0; g < k / 4; g++) {
            const uint8_t *q = src + 4 * g;
            int idx[2], c = 0;
            for (int i = 0; i < 4; i++)
                if (nonzero(q[i])) idx[c++] = i;
            // fewer than two nonzero codes: complete with the lowest other positions (whose codes are zeros)
            for (int i = 0; c < 2; i++)
                if (c == 0 || idx[0] != i) idx[c++] = i;
            if (idx[0] > idx[1]) {
                const int t = idx[0];
                idx[0] = idx[1];
                idx[1] = t;
            }
            v[2 * g] = q[idx[0]];
            v[2 * g + 1] = q[idx[1]];
            const uint8_t nib = (uint8_t)(idx[0] | (idx[1] << 2));
            uint8_t &b = m[g >> 1];
            b = (g & 1) ? (uint8_t)((b & 0x0F) | (nib << 4)) : (uint8_t)((b & 0xF0) | nib);
        }
    }
    return 0;
}

}  // namespace xtb
