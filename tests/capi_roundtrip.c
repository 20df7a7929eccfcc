/* Round trip through the C ABI from plain C: load host tables written by
 * flash_cqt_b200.tables.save_host_tables, upload them, run cqt_analysis and
 * cqt_synthesis on seeded noise and print the reconstruction SNR.
 *
 *   capi_roundtrip <tables.bin> <batch>     (exit 0 and "snr_db <value>")
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include <cuda_runtime_api.h>

#include "flash_cqt_b200.h"

#define NFIELDS 27

static void* read_field(FILE* f, size_t elem, int64_t* count) {
    if (fread(count, sizeof(int64_t), 1, f) != 1 || *count < 0) return NULL;
    void* p = malloc((size_t)(*count ? *count : 1) * elem);
    if (p && fread(p, elem, (size_t)*count, f) != (size_t)*count) {
        free(p);
        return NULL;
    }
    return p;
}

static int fail(const char* what) {
    fprintf(stderr, "%s: %s\n", what, cqt_last_error());
    return 1;
}

int main(int argc, char** argv) {
    if (argc != 3) {
        fprintf(stderr, "usage: %s <tables.bin> <batch>\n", argv[0]);
        return 2;
    }
    const int batch = atoi(argv[2]);
    FILE* f = fopen(argv[1], "rb");
    if (!f) return 2;
    /* element sizes of the fields, in the order of HOST_FIELDS */
    static const size_t elem[NFIELDS] = {4, 4, 4, 4, 4, 4, 4, 4, 4, 4, 4, 4, 4, 4,
                                         4, 4, 4, 1, 4, 4, 4, 4, 1, 4, 4, 4, 4};
    void* a[NFIELDS];
    int64_t n[NFIELDS];
    for (int i = 0; i < NFIELDS; ++i)
        if (!(a[i] = read_field(f, elem[i], &n[i]))) return 2;
    fclose(f);

    cqt_host_tables h;
    h.nbands = (int32_t)n[0];
    h.band_off = a[0]; h.band_list = a[1]; h.band_geom = a[2];
    h.ngroups = (int32_t)n[3];
    h.group_count = a[3]; h.group_roll = a[4];
    h.nclasses = (int32_t)n[5];
    h.class_len = a[5]; h.class_count = a[6]; h.class_first = a[7];
    h.ncoef = (int32_t)n[8];
    h.an_src = a[8]; h.an_gain = a[9]; h.an_seg = a[10];
    h.as_src = a[11]; h.as_gain = a[12]; h.as_seg = a[13];
    h.sy_dest = a[14]; h.sy_gre = a[15]; h.sy_gim = a[16]; h.sy_mask = a[17];
    h.sy_nplanes = *(const int32_t*)a[18];
    h.aa_dest = a[19]; h.aa_gre = a[20]; h.aa_gim = a[21]; h.aa_mask = a[22];
    h.aa_nplanes = *(const int32_t*)a[23];
    h.tw2048 = a[24]; h.tw_hi = a[25]; h.tw_lo = a[26];

    cqt_tables* t = NULL;
    if (cqt_tables_upload(&h, 0, &t)) return fail("cqt_tables_upload");
    const int ncoef = cqt_ncoef(t);
    const size_t nx = (size_t)batch * CQT_SLICE, nc = (size_t)batch * ncoef;
    float* x = malloc(nx * sizeof(float));
    float* y = malloc(nx * sizeof(float));
    uint64_t s = 0x9E3779B97F4A7C15ull;   /* xorshift noise in [-1, 1) */
    for (size_t i = 0; i < nx; ++i) {
        s ^= s << 13; s ^= s >> 7; s ^= s << 17;
        x[i] = (float)((double)(s >> 11) / 4503599627370496.0 - 1.0);
    }
    float *dx, *dy, *dc;
    void* ws;
    const size_t wsb = cqt_workspace_bytes(t, batch);
    if (cudaMalloc((void**)&dx, nx * 4) || cudaMalloc((void**)&dy, nx * 4) ||
        cudaMalloc((void**)&dc, nc * 8) || cudaMalloc(&ws, wsb))
        return 3;
    cudaMemcpy(dx, x, nx * 4, cudaMemcpyHostToDevice);
    cudaMemset(ws, 0, 256);   /* the workspace header: the wait-status word */
    if (cqt_analysis(t, dx, dc, NULL, CQT_LAYOUT_COMPLEX, batch, ws, wsb, NULL))
        return fail("cqt_analysis");
    if (cqt_synthesis(t, dc, NULL, CQT_LAYOUT_COMPLEX, dy, batch, ws, wsb, NULL))
        return fail("cqt_synthesis");
    if (cudaMemcpy(y, dy, nx * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return 3;
    double num = 0, den = 0;
    for (size_t i = 0; i < nx; ++i) {
        num += (double)x[i] * x[i];
        den += ((double)y[i] - x[i]) * ((double)y[i] - x[i]);
    }
    unsigned timeouts = 0;
    if (cqt_wait_timeouts(&timeouts) || timeouts) return fail("bounded waits");
    if (cqt_workspace_waits(ws, wsb, &timeouts, 1) || timeouts)
        return fail("bounded waits of the round trip");
    printf("snr_db %.3f\n", 10.0 * log10(num / den));
    cudaFree(dx); cudaFree(dy); cudaFree(dc); cudaFree(ws);
    cqt_tables_free(t);
    for (int i = 0; i < NFIELDS; ++i) free(a[i]);
    free(x); free(y);
    return 0;
}
