/* Test infrastructure (oracle): the INT8 row dot of the CPU restatement.
 *
 * int8_matvec_generic (ds_quantize.c:154-169) computes, per row r,
 *   y[r] = scale[r] * sum_c (q[r,c] + 128) x[c] + off[r] * sum_c x[c]
 * with both sums sequential and accumulated in one loop over c. The
 * reference is built with -O3 -march=native and gcc's default floating-point
 * contraction, so which of those multiply-adds become FMAs is gcc's choice
 * for that loop on the build host (on an AVX-512 host gcc 13 leaves the dot
 * unfused and fuses the tail; on others it fuses the dot as well). This file
 * is therefore compiled apart from ds_oracle.c, with the reference's flags
 * and contraction on, and keeps the same loop shape (one pass over c
 * carrying both sums, the same final expression), so that gcc makes the same
 * choices here and the restatement agrees with the reference bit for bit on
 * whichever machine both are built. */
#include <stdint.h>

void orc_int8_rows(float *y, const float *x, const int8_t *q, const float *scale,
                   const float *off, int row0, int row1, int in_dim) {
    for (int r = row0; r < row1; r++) {
        const int8_t *row = q + (long)r * in_dim;
        float acc = 0.0f, xsum = 0.0f;
        for (int c = 0; c < in_dim; c++) {
            acc += (float)((int)row[c] + 128) * x[c];
            xsum += x[c];
        }
        y[r] = scale[r] * acc + off[r] * xsum;
    }
}
