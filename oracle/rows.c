/*
 * rows.c -- row-batched drivers over the per-vector oracle kernels.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  The reference processes one
 * vector per call and never batches rows; these drivers call its per-vector
 * kernel once per row (the row rule of the reference CPU adapters, e.g.
 * src/backend/cpu/norm.c:12 and src/backend/cpu/softmax.c:9, applied to each
 * row of a [rows, cols] buffer), optionally over contiguous row blocks on
 * several pthreads for the all-cores CPU baseline.
 *
 * bf16 rows are widened to f32, run through the f32 kernel and rounded back
 * to bf16 (nearest-even), which is the bf16 tolerance anchor: the GPU result
 * must be within 1 bf16 ulp of exactly this.
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <dlfcn.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define ORC_ERR_OOM 7
#define ORC_ERR_INVALID_ARG 8
#define ORC_ERR_UNSUPPORTED_DTYPE 10
#define ORC_ERR_BACKEND_NOT_FOUND 14

typedef struct {
    int (*rms_norm)(size_t, const float*, const float*, float*, float);
    int (*residual_add)(size_t, const float*, const float*, float*);
    int (*gelu)(size_t, const float*, float*);
    int (*silu)(size_t, const float*, float*);
    int (*rope_gqa)(int, int, int, float*, float*, int, float);
    int (*softmax)(size_t, const float*, const float*, float*);
    int (*embedding)(const int*, int, int, const float*, float*);
} orc_table;

static const orc_table g_port = {
    orc_rms_norm_f32, orc_residual_add_f32, orc_gelu_f32, orc_silu_f32,
    orc_rope_gqa_f32, orc_softmax_f32,      orc_embedding_f32,
};
static orc_table g_ref;
static int g_ref_ok = 0;

int orc_load_ref(const char* path) {
    if (g_ref_ok) return 0;
    void* h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    if (h == NULL) return ORC_ERR_BACKEND_NOT_FOUND;
    orc_table t;
    *(void**)&t.rms_norm = dlsym(h, "tb_cpu_rms_norm_f32");
    *(void**)&t.residual_add = dlsym(h, "tb_cpu_residual_add_f32");
    *(void**)&t.gelu = dlsym(h, "tb_cpu_gelu_f32");
    *(void**)&t.silu = dlsym(h, "tb_cpu_silu_f32");
    *(void**)&t.rope_gqa = dlsym(h, "tb_cpu_rope_gqa_f32");
    *(void**)&t.softmax = dlsym(h, "tb_cpu_softmax_f32");
    *(void**)&t.embedding = dlsym(h, "tb_cpu_embedding_f32");
    if (!t.rms_norm || !t.residual_add || !t.gelu || !t.silu || !t.rope_gqa || !t.softmax ||
        !t.embedding)
        return ORC_ERR_BACKEND_NOT_FOUND;
    g_ref = t;
    g_ref_ok = 1;
    return 0;
}

int orc_ref_loaded(void) { return g_ref_ok; }

static const orc_table* pick(int impl) {
    if (impl == ORC_IMPL_PORT) return &g_port;
    if (impl == ORC_IMPL_REF && g_ref_ok) return &g_ref;
    return NULL;
}

/* ---------------------------------------------------------------------- */
/* element access                                                          */

static size_t esize(int dtype) { return dtype == ORC_BF16 ? 2 : 4; }

/* Load row `r` of a [*, cols] buffer as f32 (copy/widen into dst). */
static void load_row(int dtype, const void* base, int64_t r, int64_t cols, float* dst) {
    if (dtype == ORC_F32) {
        memcpy(dst, (const float*)base + r * cols, (size_t)cols * sizeof(float));
    } else {
        const uint16_t* s = (const uint16_t*)base + r * cols;
        for (int64_t i = 0; i < cols; i++) dst[i] = orc_bf16_to_f32(s[i]);
    }
}

static void store_row(int dtype, void* base, int64_t r, int64_t cols, const float* src) {
    if (dtype == ORC_F32) {
        memcpy((float*)base + r * cols, src, (size_t)cols * sizeof(float));
    } else {
        uint16_t* d = (uint16_t*)base + r * cols;
        for (int64_t i = 0; i < cols; i++) d[i] = orc_f32_to_bf16(src[i]);
    }
}

/* ---------------------------------------------------------------------- */
/* parallel-for over row blocks                                            */

typedef struct job job;
typedef int (*row_fn)(const job*, int64_t r0, int64_t r1, float* scratch);

struct job {
    const orc_table* t;
    int dtype;
    int64_t rows, cols;
    const void *a, *b, *c;
    void *o1, *o2;
    float f;
    int hq, hkv, hd;
    const int32_t* ids;
    int32_t* iout;
    int nscratch; /* f32 scratch rows needed per thread */
    row_fn fn;
};

typedef struct {
    const job* j;
    int64_t r0, r1;
    int rc;
} slice;

static void* run_slice(void* p) {
    slice* s = (slice*)p;
    float* scratch = NULL;
    if (s->j->nscratch > 0) {
        scratch = (float*)malloc((size_t)s->j->nscratch * (size_t)s->j->cols * sizeof(float) + 64);
        if (scratch == NULL) {
            s->rc = ORC_ERR_OOM;
            return NULL;
        }
    }
    s->rc = s->j->fn(s->j, s->r0, s->r1, scratch);
    free(scratch);
    return NULL;
}

static int run_rows(const job* j, int nthreads) {
    if (j->t == NULL) return ORC_ERR_BACKEND_NOT_FOUND;
    if (j->dtype != ORC_F32 && j->dtype != ORC_BF16) return ORC_ERR_UNSUPPORTED_DTYPE;
    if (j->rows < 0 || j->cols < 0) return ORC_ERR_INVALID_ARG;
    if (j->rows == 0) return 0;
    if (nthreads < 1) nthreads = 1;
    if ((int64_t)nthreads > j->rows) nthreads = (int)j->rows;
    if (nthreads == 1) {
        slice s = {j, 0, j->rows, 0};
        run_slice(&s);
        return s.rc;
    }
    slice* sl = (slice*)calloc((size_t)nthreads, sizeof(slice));
    pthread_t* th = (pthread_t*)calloc((size_t)nthreads, sizeof(pthread_t));
    if (sl == NULL || th == NULL) {
        free(sl);
        free(th);
        return ORC_ERR_OOM;
    }
    const int64_t base = j->rows / nthreads, extra = j->rows % nthreads;
    int64_t r = 0;
    for (int i = 0; i < nthreads; i++) {
        const int64_t n = base + (i < extra ? 1 : 0);
        sl[i].j = j;
        sl[i].r0 = r;
        sl[i].r1 = r + n;
        r += n;
        pthread_create(&th[i], NULL, run_slice, &sl[i]);
    }
    int rc = 0;
    for (int i = 0; i < nthreads; i++) {
        pthread_join(th[i], NULL);
        if (sl[i].rc != 0 && rc == 0) rc = sl[i].rc;
    }
    free(sl);
    free(th);
    return rc;
}

/* ---------------------------------------------------------------------- */
/* per-op row functions                                                     */

/* residual add (src/ops/residual.c:4) then RMSNorm (src/ops/norm.c:4) on the
 * f32 sum; h_out receives the sum (the new residual stream). */
static int rows_res_rms(const job* j, int64_t r0, int64_t r1, float* s) {
    const int64_t n = j->cols;
    float *xa = s, *ra = s + n, *h = s + 2 * n, *y = s + 3 * n, *w = s + 4 * n;
    if (j->c) load_row(j->dtype, j->c, 0, n, w);
    for (int64_t r = r0; r < r1; r++) {
        load_row(j->dtype, j->a, r, n, xa);
        load_row(j->dtype, j->b, r, n, ra);
        int rc = j->t->residual_add((size_t)n, xa, ra, h);
        if (rc) return rc;
        rc = j->t->rms_norm((size_t)n, h, j->c ? w : NULL, y, j->f);
        if (rc) return rc;
        if (j->o1) store_row(j->dtype, j->o1, r, n, h);
        store_row(j->dtype, j->o2, r, n, y);
    }
    return 0;
}

static int rows_rms(const job* j, int64_t r0, int64_t r1, float* s) {
    const int64_t n = j->cols;
    float *xa = s, *y = s + n, *w = s + 2 * n;
    if (j->b) load_row(j->dtype, j->b, 0, n, w);
    for (int64_t r = r0; r < r1; r++) {
        load_row(j->dtype, j->a, r, n, xa);
        int rc = j->t->rms_norm((size_t)n, xa, j->b ? w : NULL, y, j->f);
        if (rc) return rc;
        store_row(j->dtype, j->o1, r, n, y);
    }
    return 0;
}

static int rows_add(const job* j, int64_t r0, int64_t r1, float* s) {
    const int64_t n = j->cols;
    float *xa = s, *ra = s + n, *y = s + 2 * n;
    for (int64_t r = r0; r < r1; r++) {
        load_row(j->dtype, j->a, r, n, xa);
        load_row(j->dtype, j->b, r, n, ra);
        int rc = j->t->residual_add((size_t)n, xa, ra, y);
        if (rc) return rc;
        store_row(j->dtype, j->o1, r, n, y);
    }
    return 0;
}

static int rows_gelu(const job* j, int64_t r0, int64_t r1, float* s) {
    const int64_t n = j->cols;
    for (int64_t r = r0; r < r1; r++) {
        load_row(j->dtype, j->a, r, n, s);
        int rc = j->t->gelu((size_t)n, s, s + n);
        if (rc) return rc;
        store_row(j->dtype, j->o1, r, n, s + n);
    }
    return 0;
}

static int rows_silu(const job* j, int64_t r0, int64_t r1, float* s) {
    const int64_t n = j->cols;
    for (int64_t r = r0; r < r1; r++) {
        load_row(j->dtype, j->a, r, n, s);
        int rc = j->t->silu((size_t)n, s, s + n);
        if (rc) return rc;
        store_row(j->dtype, j->o1, r, n, s + n);
    }
    return 0;
}

/* SwiGLU composition of include/tensorbit/run/ops.hpp:246-248:
 * silu(gate) with the table's silu, then *= up. */
static int rows_swiglu(const job* j, int64_t r0, int64_t r1, float* s) {
    const int64_t n = j->cols;
    float *g = s, *u = s + n, *o = s + 2 * n;
    for (int64_t r = r0; r < r1; r++) {
        load_row(j->dtype, j->a, r, n, g);
        load_row(j->dtype, j->b, r, n, u);
        int rc = j->t->silu((size_t)n, g, o);
        if (rc) return rc;
        for (int64_t i = 0; i < n; i++) o[i] *= u[i];
        store_row(j->dtype, j->o1, r, n, o);
    }
    return 0;
}

/* RoPE: row r of q is [hq, hd], row r of k is [hkv, hd]; rotated in place at
 * positions[r] (tb_cpu_rope_gqa_f32, src/ops/rope.c:43, once per token). */
static int rows_rope(const job* j, int64_t r0, int64_t r1, float* s) {
    const int64_t qn = (int64_t)j->hq * j->hd, kn = (int64_t)j->hkv * j->hd;
    float *qa = s, *ka = s + qn;
    for (int64_t r = r0; r < r1; r++) {
        load_row(j->dtype, j->o1, r, qn, qa);
        load_row(j->dtype, j->o2, r, kn, ka);
        int rc = j->t->rope_gqa(j->hq, j->hkv, j->hd, qa, ka, j->ids[r], j->f);
        if (rc) return rc;
        store_row(j->dtype, j->o1, r, qn, qa);
        store_row(j->dtype, j->o2, r, kn, ka);
    }
    return 0;
}

static int rows_softmax(const job* j, int64_t r0, int64_t r1, float* s) {
    const int64_t n = j->cols;
    float *xa = s, *m = s + n, *y = s + 2 * n;
    for (int64_t r = r0; r < r1; r++) {
        load_row(j->dtype, j->a, r, n, xa);
        if (j->b) load_row(j->dtype, j->b, r, n, m);
        int rc = j->t->softmax((size_t)n, xa, j->b ? m : NULL, y);
        if (rc) return rc;
        store_row(j->dtype, j->o1, r, n, y);
    }
    return 0;
}

static int rows_argmax(const job* j, int64_t r0, int64_t r1, float* s) {
    const int64_t n = j->cols;
    for (int64_t r = r0; r < r1; r++) {
        const float* row;
        if (j->dtype == ORC_F32) {
            row = (const float*)j->a + r * n;
        } else {
            load_row(j->dtype, j->a, r, n, s);
            row = s;
        }
        j->iout[r] = orc_argmax_f32(row, (int)n);
    }
    return 0;
}

/* Embedding: the per-call kernel takes all ids at once; one call per block of
 * tokens keeps it a single call per thread as the reference would make. */
static int rows_embedding(const job* j, int64_t r0, int64_t r1, float* s) {
    (void)s;
    const int64_t d = j->cols;
    if (j->dtype == ORC_F32) {
        return j->t->embedding(j->ids + r0, (int)(r1 - r0), (int)d, (const float*)j->a,
                               (float*)j->o1 + r0 * d);
    }
    /* bf16 tables: the gather is a byte copy of whole rows. */
    for (int64_t r = r0; r < r1; r++) {
        memcpy((uint16_t*)j->o1 + r * d, (const uint16_t*)j->a + (int64_t)j->ids[r] * d,
               (size_t)d * 2);
    }
    return 0;
}

/* ---------------------------------------------------------------------- */
/* entry points                                                             */

static job mk(int impl, int dtype, int64_t rows, int64_t cols, row_fn fn, int nscratch) {
    job j;
    memset(&j, 0, sizeof j);
    j.t = pick(impl);
    j.dtype = dtype;
    j.rows = rows;
    j.cols = cols;
    j.fn = fn;
    j.nscratch = nscratch;
    return j;
}

int orc_rows_residual_rms_norm(int impl, int dtype, int64_t rows, int64_t cols, const void* x,
                               const void* residual, const void* weight, void* h_out, void* y,
                               float eps, int nthreads) {
    job j = mk(impl, dtype, rows, cols, rows_res_rms, 5);
    j.a = x;
    j.b = residual;
    j.c = weight;
    j.o1 = h_out;
    j.o2 = y;
    j.f = eps;
    return run_rows(&j, nthreads);
}

int orc_rows_rms_norm(int impl, int dtype, int64_t rows, int64_t cols, const void* x,
                      const void* weight, void* y, float eps, int nthreads) {
    job j = mk(impl, dtype, rows, cols, rows_rms, 3);
    j.a = x;
    j.b = weight;
    j.o1 = y;
    j.f = eps;
    return run_rows(&j, nthreads);
}

int orc_rows_residual_add(int impl, int dtype, int64_t rows, int64_t cols, const void* x,
                          const void* residual, void* y, int nthreads) {
    job j = mk(impl, dtype, rows, cols, rows_add, 3);
    j.a = x;
    j.b = residual;
    j.o1 = y;
    return run_rows(&j, nthreads);
}

int orc_rows_gelu(int impl, int dtype, int64_t rows, int64_t cols, const void* x, void* y,
                  int nthreads) {
    job j = mk(impl, dtype, rows, cols, rows_gelu, 2);
    j.a = x;
    j.o1 = y;
    return run_rows(&j, nthreads);
}

int orc_rows_silu(int impl, int dtype, int64_t rows, int64_t cols, const void* x, void* y,
                  int nthreads) {
    job j = mk(impl, dtype, rows, cols, rows_silu, 2);
    j.a = x;
    j.o1 = y;
    return run_rows(&j, nthreads);
}

int orc_rows_swiglu(int impl, int dtype, int64_t rows, int64_t cols, const void* gate,
                    const void* up, void* out, int nthreads) {
    job j = mk(impl, dtype, rows, cols, rows_swiglu, 3);
    j.a = gate;
    j.b = up;
    j.o1 = out;
    return run_rows(&j, nthreads);
}

int orc_rows_rope(int impl, int dtype, int64_t rows, int n_q_heads, int n_kv_heads, int head_dim,
                  void* q, void* k, const int32_t* positions, float theta, int nthreads) {
    if (n_q_heads < 0 || n_kv_heads < 0 || head_dim < 0 || positions == NULL)
        return ORC_ERR_INVALID_ARG;
    const int64_t widest = (int64_t)(n_q_heads > n_kv_heads ? n_q_heads : n_kv_heads) * head_dim;
    job j = mk(impl, dtype, rows, widest, rows_rope, 2);
    j.o1 = q;
    j.o2 = k;
    j.hq = n_q_heads;
    j.hkv = n_kv_heads;
    j.hd = head_dim;
    j.ids = positions;
    j.f = theta;
    return run_rows(&j, nthreads);
}

int orc_rows_softmax(int impl, int dtype, int64_t rows, int64_t cols, const void* x,
                     const void* mask, void* y, int nthreads) {
    job j = mk(impl, dtype, rows, cols, rows_softmax, 3);
    j.a = x;
    j.b = mask;
    j.o1 = y;
    return run_rows(&j, nthreads);
}

int orc_rows_argmax(int impl, int dtype, int64_t rows, int64_t cols, const void* x, int32_t* out,
                    int nthreads) {
    if (cols < 1) return ORC_ERR_INVALID_ARG;
    job j = mk(impl, dtype, rows, cols, rows_argmax, dtype == ORC_BF16 ? 1 : 0);
    j.a = x;
    j.iout = out;
    return run_rows(&j, nthreads);
}

int orc_rows_embedding(int impl, int dtype, int64_t n_tokens, int64_t dim, const int32_t* ids,
                       const void* table, void* y, int nthreads) {
    job j = mk(impl, dtype, n_tokens, dim, rows_embedding, 0);
    j.a = table;
    j.o1 = y;
    j.ids = ids;
    return run_rows(&j, nthreads);
}
