/* FP64 dense paged attention in C.  TEST INFRASTRUCTURE ONLY.
 *
 * Restates dense_attention + gather_cache of ensigncode/paged-decode-lab
 * (src/paged_decode/oracle.py:50-71): for every (sequence b, query head h)
 * gather the live tokens t < lengths[b] through page table row b
 * (physical page table[b][t / T], slot t % T, KV head h / (Hq / Hkv)),
 * score them against q[b][h] in double precision scaled by 1/sqrt(D),
 * softmax with max subtraction, and average the value rows.  A zero-length
 * sequence yields a zero row.  Inputs are float16 or float32; output is
 * float64 [B, Hq, D].
 *
 * Work is split over threads by (sequence, KV head) units so every K/V row
 * of a unit is read once for the whole query-head group.  The product never
 * links this file: it is the checker for large parity cases and the timed
 * CPU baseline.
 */
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    const void *q, *k, *v;
    int elem_bytes;
    const int32_t *table, *lengths;
    int batch, q_heads, kv_heads, head_dim, page_size, table_width;
    double *out;
    atomic_int next_unit;
    atomic_int failed;
} job_t;

static inline double load_elem(const void *base, int64_t index, int elem_bytes) {
    if (elem_bytes == 2) return (double)((const _Float16 *)base)[index];
    return (double)((const float *)base)[index];
}

static int run_unit(job_t *job, int unit) {
    const int b = unit / job->kv_heads;
    const int kvh = unit % job->kv_heads;
    const int group = job->q_heads / job->kv_heads;
    const int D = job->head_dim;
    const int64_t length = job->lengths[b];
    double *out_rows = job->out + ((int64_t)b * job->q_heads + (int64_t)kvh * group) * D;
    memset(out_rows, 0, sizeof(double) * (size_t)group * D);
    if (length == 0) return 0;

    double *qd = malloc(sizeof(double) * (size_t)group * D);
    double *scores = malloc(sizeof(double) * (size_t)group * length);
    double *row = malloc(sizeof(double) * (size_t)D);
    if (!qd || !scores || !row) { free(qd); free(scores); free(row); return -1; }

    const double inv_sqrt_d = 1.0 / sqrt((double)D);
    for (int g = 0; g < group; ++g)
        for (int d = 0; d < D; ++d)
            qd[g * D + d] = load_elem(job->q, ((int64_t)b * job->q_heads + kvh * group + g) * D + d,
                                      job->elem_bytes);

    /* scores[g][t] = <q_g, K[t]> / sqrt(D) */
    for (int64_t t = 0; t < length; ++t) {
        const int64_t page = job->table[(int64_t)b * job->table_width + t / job->page_size];
        const int64_t base = ((page * job->page_size + t % job->page_size) * job->kv_heads + kvh) * D;
        for (int d = 0; d < D; ++d) row[d] = load_elem(job->k, base + d, job->elem_bytes);
        for (int g = 0; g < group; ++g) {
            double acc = 0.0;
            for (int d = 0; d < D; ++d) acc += qd[g * D + d] * row[d];
            scores[g * length + t] = acc * inv_sqrt_d;
        }
    }
    /* weights = exp(s - max); the division by their sum comes last */
    double *sums = qd; /* q no longer needed: reuse as per-head sums */
    for (int g = 0; g < group; ++g) {
        double top = -INFINITY;
        for (int64_t t = 0; t < length; ++t) top = fmax(top, scores[g * length + t]);
        double total = 0.0;
        for (int64_t t = 0; t < length; ++t) {
            const double w = exp(scores[g * length + t] - top);
            scores[g * length + t] = w;
            total += w;
        }
        sums[g] = total;
    }
    for (int64_t t = 0; t < length; ++t) {
        const int64_t page = job->table[(int64_t)b * job->table_width + t / job->page_size];
        const int64_t base = ((page * job->page_size + t % job->page_size) * job->kv_heads + kvh) * D;
        for (int d = 0; d < D; ++d) row[d] = load_elem(job->v, base + d, job->elem_bytes);
        for (int g = 0; g < group; ++g) {
            const double w = scores[g * length + t];
            double *o = out_rows + (int64_t)g * D;
            for (int d = 0; d < D; ++d) o[d] += w * row[d];
        }
    }
    for (int g = 0; g < group; ++g)
        for (int d = 0; d < D; ++d) out_rows[(int64_t)g * D + d] /= sums[g];
    free(qd); free(scores); free(row);
    return 0;
}

static void *worker(void *arg) {
    job_t *job = arg;
    const int units = job->batch * job->kv_heads;
    for (;;) {
        const int unit = atomic_fetch_add(&job->next_unit, 1);
        if (unit >= units) break;
        if (run_unit(job, unit) != 0) atomic_store(&job->failed, 1);
    }
    return NULL;
}

/* Returns 0 on success, -1 on bad arguments or allocation failure. */
int pdo_dense_attention(const void *q, const void *k, const void *v, int elem_bytes,
                        const int32_t *table, const int32_t *lengths, int batch, int q_heads,
                        int kv_heads, int head_dim, int page_size, int table_width,
                        double *out, int threads) {
    if (!q || !k || !v || !table || !lengths || !out) return -1;
    if ((elem_bytes != 2 && elem_bytes != 4) || batch <= 0 || q_heads <= 0 || kv_heads <= 0 ||
        q_heads % kv_heads || head_dim <= 0 || page_size <= 0 || table_width < 0)
        return -1;
    job_t job = {q, k, v, elem_bytes, table, lengths, batch, q_heads, kv_heads, head_dim,
                 page_size, table_width, out, 0, 0};
    atomic_init(&job.next_unit, 0);
    atomic_init(&job.failed, 0);
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t ids[256];
    int started = 0;
    for (int i = 1; i < threads; ++i)
        if (pthread_create(&ids[started], NULL, worker, &job) == 0) ++started;
    worker(&job);
    for (int i = 0; i < started; ++i) pthread_join(ids[i], NULL);
    return atomic_load(&job.failed) ? -1 : 0;
}
