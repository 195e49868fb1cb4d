/* par.h — a pthreads parallel-for for the oracle (test infrastructure only). */
#ifndef AJI_ORACLE_PAR_H
#define AJI_ORACLE_PAR_H

/* Runs fn(ctx, i) for i in [0, n) on nthreads threads (<= 0: all online cores), items handed
 * out one at a time from a shared counter. Each item is computed exactly as on one thread. */
void orc_par_for(int n, int nthreads, void (*fn)(void *ctx, int i), void *ctx);
int orc_cores(void);

#endif
