/*
 * eii_check VECTORDIR [MODELDIR]
 *
 * Drop-in for the reference's conformance checkers (c/intref.c:214-258, cuda/intref.cu:262-306):
 * reads MODELDIR/model.bin (MODELDIR defaults to VECTORDIR), VECTORDIR/ids.i64 and the expected
 * states exported by python/export_vectors.py, runs the B200 engine through the C ABI, and
 * prints the same lines: "  MISMATCH ...", "layer %2d: exact|DIFFERS", "logits: exact|DIFFERS",
 * then "ALL STATES EXACT (...)" or "FAIL (...)".  Exit status 0 exact, 1 mismatch, 2 I/O error,
 * 3 CUDA error (as the reference programs), 4 other engine error.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "eii.h"

enum { V = 49152, D = 576, NL = 30 };

static void* read_file(const char* dir, const char* name, size_t* nbytes) {
    char path[4096];
    snprintf(path, sizeof path, "%s/%s", dir, name);
    FILE* f = fopen(path, "rb");
    if (!f) { perror(path); exit(2); }
    fseek(f, 0, SEEK_END);
    long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    void* p = malloc(n > 0 ? (size_t)n : 1);
    if (!p || fread(p, 1, (size_t)n, f) != (size_t)n) { fprintf(stderr, "short read\n"); exit(2); }
    fclose(f);
    *nbytes = (size_t)n;
    return p;
}

static size_t compare32(const char* name, const int32_t* got, const int32_t* exp, size_t n) {
    size_t bad = 0, first = (size_t)-1;
    for (size_t i = 0; i < n; i++)
        if (got[i] != exp[i]) { if (!bad) first = i; bad++; }
    if (bad)
        printf("  MISMATCH %-12s %zu of %zu, first at %zu (got %d expected %d)\n", name, bad, n, first, got[first], exp[first]);
    return bad;
}

static int exit_for(int rc) { return rc == EII_ERR_IO ? 2 : rc == EII_ERR_CUDA ? 3 : 4; }

int main(int argc, char** argv) {
    if (argc < 2) { fprintf(stderr, "usage: eii_check VECTORDIR [MODELDIR]\n"); return 2; }
    const char* vdir = argv[1];
    const char* mdir = argc > 2 ? argv[2] : argv[1];
    char path[4096];
    snprintf(path, sizeof path, "%s/model.bin", mdir);
    size_t nb;
    int64_t* ids = (int64_t*)read_file(vdir, "ids.i64", &nb);
    const int T = (int)(nb / 8);
    if (T < 1 || T > 512) { fprintf(stderr, "T = %d outside [1, 512]\n", T); return 2; }
    int32_t* exp_embed = (int32_t*)read_file(vdir, "exp_embed.i32", &nb);
    if (nb != (size_t)T * D * 4) { fprintf(stderr, "short read\n"); return 2; }
    int32_t* exp_res = (int32_t*)read_file(vdir, "exp_resid_out.i32", &nb);
    if (nb != (size_t)NL * T * D * 4) { fprintf(stderr, "short read\n"); return 2; }
    int32_t* exp_log = (int32_t*)read_file(vdir, "exp_logits.i32", &nb);
    if (nb != (size_t)T * V * 4) { fprintf(stderr, "short read\n"); return 2; }

    eii_engine* e = NULL;
    int rc = eii_open(path, 0, &e);
    if (rc != EII_OK) { fprintf(stderr, "%s\n", eii_last_error()); return exit_for(rc); }
    int32_t* embed = (int32_t*)malloc((size_t)T * D * 4);
    int32_t* res = (int32_t*)malloc((size_t)NL * T * D * 4);
    int32_t* logits = (int32_t*)malloc((size_t)T * V * 4);
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    rc = eii_forward(e, ids, 1, T, embed, res, logits, NULL);
    if (rc != EII_OK) { fprintf(stderr, "%s\n", eii_last_error()); eii_close(e); return exit_for(rc); }
    size_t total_bad = compare32("embed", embed, exp_embed, (size_t)T * D);
    for (int l = 0; l < NL && !total_bad; l++) {
        size_t bad = compare32("resid_out", res + (size_t)l * T * D, exp_res + (size_t)l * T * D, (size_t)T * D);
        printf("layer %2d: %s\n", l, bad ? "DIFFERS" : "exact");
        total_bad += bad;
    }
    if (!total_bad) {
        total_bad += compare32("logits", logits, exp_log, (size_t)T * V);
        printf("logits: %s\n", total_bad ? "DIFFERS" : "exact");
    }
    clock_gettime(CLOCK_MONOTONIC, &t1);
    const double s = (double)(t1.tv_sec - t0.tv_sec) + 1e-9 * (double)(t1.tv_nsec - t0.tv_nsec);
    printf("%s (%d tokens, %.2f s on device incl. comparisons)\n", total_bad ? "FAIL" : "ALL STATES EXACT", T, s);
    eii_close(e);
    return total_bad ? 1 : 0;
}
