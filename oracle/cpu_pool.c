/*
 * cpu_pool.c -- row-partitioned threaded matvec for the CPU baseline.
 * TEST / BASELINE INFRASTRUCTURE ONLY.
 *
 * Mirrors the reference's CPU thread pool (src/minicpmo/qwen3.uya:1247-1499):
 * participant p of P computes rows [out*p/P, out*(p+1)/P), participant 0 is
 * the calling thread, workers spin with yields between tasks.  Each part
 * calls the reference's own native matvec, minicpmo_cpu_matvec_range
 * (src/minicpmo/cpu_kernels.c:791-851), when oracle/_ref/libref_cpu.so is
 * available ("reference" baseline); otherwise the oracle restatement
 * orc_matvec_f32 ("port" baseline).
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <dlfcn.h>
#include <pthread.h>
#include <sched.h>
#include <stdlib.h>
#include <string.h>

typedef int (*ref_matvec_range_fn)(float *, const uint8_t *, int, const float *, size_t, size_t, size_t);

typedef struct orc_pool {
    int threads;
    pthread_t *tids;
    void *ref_lib;
    ref_matvec_range_fn ref_range;
    /* task */
    volatile unsigned long seq;
    volatile unsigned long done;
    volatile int stop;
    int dtype;
    const uint8_t *w;
    size_t rows, cols, row_bytes;
    const float *x;
    const uint8_t *xq;  /* Q8_1 task: the quantised activations */
    int q8_1_order;     /* Q8_1 task: 1 device order, 0 natural order; -1 an f32 task */
    float *y;
    volatile int failed;
} orc_pool;

typedef struct { orc_pool *pool; int id; } worker_arg;

static void do_part(orc_pool *p, int part) {
    size_t start = p->rows * (size_t) part / (size_t) p->threads;
    size_t end = p->rows * (size_t) (part + 1) / (size_t) p->threads;
    if (end <= start) return;
    if (p->q8_1_order >= 0) {
        /* every row is computed on its own, so a row range gives the rows'
         * bits of the whole-matrix call */
        const uint8_t *w = p->w + start * p->row_bytes;
        if (!(p->q8_1_order ? orc_matvec_q8_1_dev(p->dtype, w, end - start, p->cols, p->xq, p->y + start)
                            : orc_matvec_q8_1(p->dtype, w, end - start, p->cols, p->xq, p->y + start)))
            p->failed = 1;
    } else if (p->ref_range) {
        if (!p->ref_range(p->y, p->w, p->dtype, p->x, p->cols, start, end)) p->failed = 1;
    } else {
        if (!orc_matvec_f32(p->dtype, p->w + start * p->row_bytes, end - start, p->cols, p->x, p->y + start)) p->failed = 1;
    }
}

static void *worker_main(void *arg) {
    worker_arg *wa = (worker_arg *) arg;
    orc_pool *p = wa->pool;
    unsigned long seen = 0;
    int id = wa->id;
    free(wa);
    for (;;) {
        unsigned long now;
        if (p->stop) return NULL;
        now = __atomic_load_n(&p->seq, __ATOMIC_ACQUIRE);
        if (now == seen) { sched_yield(); continue; }
        do_part(p, id);
        __atomic_fetch_add(&p->done, 1, __ATOMIC_ACQ_REL);
        seen = now;
    }
}

void *orc_pool_create(int threads, const char *ref_cpu_so) {
    orc_pool *p = (orc_pool *) calloc(1, sizeof(orc_pool));
    int i;
    if (!p) return NULL;
    if (threads < 1) threads = 1;
    p->threads = threads;
    if (ref_cpu_so && ref_cpu_so[0]) {
        p->ref_lib = dlopen(ref_cpu_so, RTLD_NOW | RTLD_LOCAL);
        if (p->ref_lib) p->ref_range = (ref_matvec_range_fn) dlsym(p->ref_lib, "minicpmo_cpu_matvec_range");
    }
    p->tids = (pthread_t *) calloc((size_t) threads, sizeof(pthread_t));
    for (i = 1; i < threads; ++i) {
        worker_arg *wa = (worker_arg *) malloc(sizeof(worker_arg));
        wa->pool = p;
        wa->id = i;
        pthread_create(&p->tids[i], NULL, worker_main, wa);
    }
    return p;
}

int orc_pool_is_reference(void *pool) { return pool && ((orc_pool *) pool)->ref_range != NULL; }

static int run_task(orc_pool *p);

int orc_pool_matvec(void *user, int dtype, const uint8_t *w, size_t rows, size_t cols, const float *x, float *y) {
    orc_pool *p = (orc_pool *) user;
    p->dtype = dtype; p->w = w; p->rows = rows; p->cols = cols; p->x = x; p->y = y;
    p->xq = NULL; p->q8_1_order = -1;
    return run_task(p);
}

int orc_pool_matvec_q8_1(void *user, int order, int dtype, const uint8_t *w, size_t rows, size_t cols,
                         const uint8_t *xq, float *y) {
    orc_pool *p = (orc_pool *) user;
    p->dtype = dtype; p->w = w; p->rows = rows; p->cols = cols; p->x = NULL; p->y = y;
    p->xq = xq; p->q8_1_order = order ? 1 : 0;
    return run_task(p);
}

static int run_task(orc_pool *p) {
    unsigned long target;
    p->row_bytes = orc_row_bytes(p->dtype, p->cols);
    p->failed = 0;
    if (p->row_bytes == 0) return 0;
    if (p->threads == 1) { do_part(p, 0); return !p->failed; }
    __atomic_store_n(&p->done, 0, __ATOMIC_RELEASE);
    __atomic_fetch_add(&p->seq, 1, __ATOMIC_ACQ_REL);
    do_part(p, 0);
    target = (unsigned long) (p->threads - 1);
    while (__atomic_load_n(&p->done, __ATOMIC_ACQUIRE) < target) sched_yield();
    return !p->failed;
}

void orc_pool_destroy(void *pool) {
    orc_pool *p = (orc_pool *) pool;
    int i;
    if (!p) return;
    p->stop = 1;
    for (i = 1; i < p->threads; ++i) pthread_join(p->tids[i], NULL);
    /* the reference library stays mapped until the process exits: a later
     * pool reuses it, and the mapping shows which native code ran */
    free(p->tids);
    free(p);
}

void orc_state_attach_pool(orc_state *st, void *pool) {
    st->matvec = pool ? orc_pool_matvec : NULL;
    st->matvec_user = pool;
}
