/* par.c — see par.h. */
#include "par.h"

#include <pthread.h>
#include <stdatomic.h>
#include <unistd.h>

struct par_state {
    atomic_int next;
    int n;
    void (*fn)(void *, int);
    void *ctx;
};

static void *worker(void *arg)
{
    struct par_state *s = (struct par_state *)arg;
    for (;;) {
        const int i = atomic_fetch_add(&s->next, 1);
        if (i >= s->n) break;
        s->fn(s->ctx, i);
    }
    return 0;
}

int orc_cores(void)
{
    const long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

void orc_par_for(int n, int nthreads, void (*fn)(void *ctx, int i), void *ctx)
{
    if (nthreads <= 0) nthreads = orc_cores();
    if (nthreads > 256) nthreads = 256;
    if (nthreads > n) nthreads = n;
    struct par_state s;
    atomic_init(&s.next, 0);
    s.n = n;
    s.fn = fn;
    s.ctx = ctx;
    if (nthreads <= 1) {
        worker(&s);
        return;
    }
    pthread_t th[256];
    int started = 0;
    for (int t = 1; t < nthreads; t++)
        if (pthread_create(&th[started], 0, worker, &s) == 0) started++;
    worker(&s);
    for (int t = 0; t < started; t++) pthread_join(th[t], 0);
}
