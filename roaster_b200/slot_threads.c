/*
 * slot_threads.c -- native slot threads driving the cross-slot batched step.
 *
 * The reference serves each slot's request on its own pthread (slots.c run_impl), and every
 * token of every slot passes through step_forward (slots.c:864-880). This driver plays those
 * threads against libroaster_b200's step group: thread i is member ids[i]; per token it calls
 * kernel_step_group_begin, one kernel_step_group_matvec per layer (site = layer, the slot's own
 * projection jobs of that layer), kernel_step_group_end. It exists so that a measurement of the
 * group sees native threads as slots.c would run them, not an interpreter's lock. It makes no
 * CUDA call of its own.
 *
 * Built by roaster_b200/build.py into libslot_threads.so (linked against libroaster_b200.so).
 */
#include <pthread.h>
#include <stdlib.h>

#include "roaster_cuda.h"

typedef struct {
    KernelStepGroup *g;
    int member, rounds, sites;
    const KernelCudaMatvecJob *jobs;   /* this slot's jobs, sites after one another */
    const int *per_site;               /* jobs of each site */
    int rc;
} SlotArg;

static void *slot_main(void *p)
{
    SlotArg *a = (SlotArg *)p;
    a->rc = 0;
    for (int r = 0; r < a->rounds && a->rc == 0; r++) {
        if (kernel_step_group_begin(a->g, a->member) < 1) {
            a->rc = -1;
            break;
        }
        const KernelCudaMatvecJob *j = a->jobs;
        for (int s = 0; s < a->sites; s++) {
            if (kernel_step_group_matvec(a->g, a->member, s, j, a->per_site[s]) != 0)
                a->rc = -1;
            j += a->per_site[s];
        }
        if (kernel_step_group_end(a->g, a->member) != 0)
            a->rc = -1;
    }
    return NULL;
}

/* n slot threads, each `rounds` tokens over `sites` layers. jobs = n blocks of `total` jobs
 * (total = sum of per_site), block i for member ids[i]. 0 when every call of every thread
 * returned 0, else -1 (kernel_cuda_last_error has the last message). */
int slot_threads_run(KernelStepGroup *g, int n, const int *ids, int rounds, int sites, const int *per_site,
                     const KernelCudaMatvecJob *jobs, int total)
{
    if (!g || n < 1 || !ids || rounds < 1 || sites < 1 || !per_site || !jobs || total < 1)
        return -1;
    pthread_t *th = (pthread_t *)calloc((size_t)n, sizeof(pthread_t));
    SlotArg *args = (SlotArg *)calloc((size_t)n, sizeof(SlotArg));
    if (!th || !args) {
        free(th);
        free(args);
        return -1;
    }
    int started = 0, rc = 0;
    for (int i = 0; i < n; i++) {
        args[i] = (SlotArg){g, ids[i], rounds, sites, jobs + (size_t)i * (size_t)total, per_site, 0};
        if (pthread_create(&th[i], NULL, slot_main, &args[i]) != 0) {
            rc = -1;
            break;
        }
        started++;
    }
    for (int i = 0; i < started; i++) {
        pthread_join(th[i], NULL);
        if (args[i].rc != 0)
            rc = -1;
    }
    free(th);
    free(args);
    return rc;
}
