/*
 * ffa_oracle.c -- CPU restatement of the reference aligner's conventional
 * path.  TEST INFRASTRUCTURE ONLY (see ffa_oracle.h): the checker, never the
 * thing measured or shipped.
 *
 * Every step cites the reference file:line it restates
 * (src/fast_forced_aligner/csrc/alignment.cu of brthor/fast-forced-aligner).
 * Build with -ffp-contract=off and without -ffast-math so each DP cell is one
 * IEEE fp32 round-to-nearest addition, as in the reference (which builds with
 * --fmad=false, alignment.py:60).
 */
#include "ffa_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

typedef struct {
  const ffa_oracle_record* records;
  int64_t B;
  int check_inputs;
  const uint8_t* validity;
  const int64_t* offsets;  /* frame offset of each record in the outputs */
  const int64_t* order;    /* records, most expensive first */
  int64_t* labels;
  float* scores;
  int32_t* status;
  float* objective;
  atomic_long next;
  atomic_int error;
} job_t;

static void fail_record(int64_t T, int64_t* labels, float* scores) {
  /* Failed records: -1 labels, -inf scores (alignment.cu:650-652). */
  for (int64_t t = 0; t < T; ++t) {
    labels[t] = -1;
    scores[t] = -INFINITY;
  }
}

/* Returns 0 on success, -1 when an unchecked target ID is out of range. */
static int align_record(const ffa_oracle_record* r, int check_inputs,
                        int masked_out, int64_t* labels, float* scores,
                        int32_t* status_out, float* objective_out) {
  const int64_t T = r->T, V = r->V, U = r->U, blank = r->blank;
  const float* e = r->emissions;
  const int64_t* tokens = r->targets;

  /* Mask first, then target validation overrides it (alignment.cu:836,
   * 852-874): invalid IDs -> 3, else U + adjacent repeats > T -> 4. */
  int status = masked_out ? FFA_ORACLE_MASKED : FFA_ORACLE_OK;
  if (check_inputs) {
    int bad = 0;
    int64_t repeats = 0;
    for (int64_t k = 0; k < U; ++k) {
      const int64_t token = tokens[k];
      if (token < 0 || token >= V || token == blank) bad = 1;
      if (k > 0 && token == tokens[k - 1]) ++repeats;
    }
    if (bad) status = FFA_ORACLE_BAD_TARGET;
    else if (U + repeats > T) status = FFA_ORACLE_TOO_FEW_FRAMES;
  } else {
    for (int64_t k = 0; k < U; ++k)
      if (tokens[k] < 0 || tokens[k] >= V) return -1;
  }
  if (status >= FFA_ORACLE_MASKED) {
    /* Statuses >= 2 skip every DP stage; objective stays -inf
     * (alignment.cu:837, 361). */
    *status_out = status;
    *objective_out = -INFINITY;
    fail_record(T, labels, scores);
    return 0;
  }

  /* Expanded CTC states: blank at even s, target (s-1)/2 at odd s
   * (alignment.cu:856-857). */
  const int64_t S = 2 * U + 1;
  int64_t* l = (int64_t*)malloc(sizeof(int64_t) * (size_t)S);
  float* prev = (float*)malloc(sizeof(float) * (size_t)S);
  float* next = (float*)malloc(sizeof(float) * (size_t)S);
  /* Two bits per cell hold the jump 0 (stay), 1 (step) or 2 (skip). */
  const size_t bp_bytes = (size_t)((T * S + 3) / 4);
  uint8_t* bp = (uint8_t*)calloc(bp_bytes, 1);
  if (!l || !prev || !next || !bp) {
    free(l); free(prev); free(next); free(bp);
    return -2;
  }
  for (int64_t s = 0; s < S; ++s) l[s] = (s & 1) ? tokens[s / 2] : blank;

  /* Init at frame 0: alpha[s] = e[0, l[s]] for s < 2, else -inf;
   * bp[0, s] = 0 (alignment.cu:409-410). */
  for (int64_t s = 0; s < S; ++s) prev[s] = s < 2 ? e[l[s]] : -INFINITY;

  /* Recurrence (alignment.cu:414-429): stay, then step if strictly greater,
   * then skip if strictly greater and legal; one fp32 add per cell. */
  for (int64_t t = 1; t < T; ++t) {
    const float* row = e + t * V;
    for (int64_t s = 0; s < S; ++s) {
      float best = prev[s];
      unsigned jump = 0;
      if (s >= 1 && prev[s - 1] > best) { best = prev[s - 1]; jump = 1; }
      if (s >= 2 && l[s] != blank && l[s] != l[s - 2] && prev[s - 2] > best) {
        best = prev[s - 2];
        jump = 2;
      }
      next[s] = best + row[l[s]];
      const int64_t cell = t * S + s;
      bp[cell >> 2] |= (uint8_t)(jump << (2 * (cell & 3)));
    }
    float* swap = prev; prev = next; next = swap;
  }

  /* Terminal: S-1 unless S > 1 and alpha[S-2] >= alpha[S-1]
   * (alignment.cu:497-499); status from finiteness (alignment.cu:507-510). */
  int64_t terminal = S - 1;
  if (S > 1 && prev[S - 2] >= prev[S - 1]) terminal = S - 2;
  const float objective = prev[terminal];
  *objective_out = objective;
  if (!isfinite(objective)) {
    *status_out = FFA_ORACLE_NO_PATH;
    fail_record(T, labels, scores);
  } else {
    *status_out = FFA_ORACLE_OK;
    /* Traceback path[t] = s; s -= bp[t, s]; then labels and selected scores
     * (alignment.cu:654-666). */
    int64_t s = terminal;
    for (int64_t t = T - 1; t >= 0; --t) {
      const int64_t label = l[s];
      labels[t] = label;
      scores[t] = e[t * V + label];
      const int64_t cell = t * S + s;
      s -= (bp[cell >> 2] >> (2 * (cell & 3))) & 3;
    }
  }
  free(l); free(prev); free(next); free(bp);
  return 0;
}

static void* worker(void* arg) {
  job_t* job = (job_t*)arg;
  for (;;) {
    const long k = atomic_fetch_add(&job->next, 1);
    if (k >= job->B) break;
    const int64_t i = job->order[k];
    const int masked = job->validity != NULL && !job->validity[i];
    const int rc = align_record(&job->records[i], job->check_inputs, masked,
                                job->labels + job->offsets[i],
                                job->scores + job->offsets[i],
                                job->status + i, job->objective + i);
    if (rc) atomic_store(&job->error, rc);
  }
  return NULL;
}

static int cmp_cost_desc(const void* a, const void* b, void* ctx) {
  const ffa_oracle_record* r = (const ffa_oracle_record*)ctx;
  const int64_t i = *(const int64_t*)a, j = *(const int64_t*)b;
  const int64_t ci = r[i].T * (2 * r[i].U + 1), cj = r[j].T * (2 * r[j].U + 1);
  return ci < cj ? 1 : (ci > cj ? -1 : (i > j) - (i < j));
}

int ffa_oracle_align(const ffa_oracle_record* records, int64_t B,
                     int check_inputs, const uint8_t* validity, int threads,
                     int64_t* labels, float* scores, int32_t* status,
                     float* objective) {
  if (B <= 0 || !records || !labels || !scores || !status || !objective) return -1;
  for (int64_t i = 0; i < B; ++i) {
    const ffa_oracle_record* r = &records[i];
    if (r->T <= 0 || r->V <= 0 || r->U < 0 || !r->emissions ||
        (r->U > 0 && !r->targets) || r->blank < 0 || r->blank >= r->V)
      return -1;
  }
  int64_t* offsets = (int64_t*)malloc(sizeof(int64_t) * (size_t)B);
  int64_t* order = (int64_t*)malloc(sizeof(int64_t) * (size_t)B);
  if (!offsets || !order) { free(offsets); free(order); return -2; }
  int64_t total = 0;
  for (int64_t i = 0; i < B; ++i) { offsets[i] = total; total += records[i].T; order[i] = i; }
  qsort_r(order, (size_t)B, sizeof(int64_t), cmp_cost_desc, (void*)records);

  if (threads <= 0) threads = (int)sysconf(_SC_NPROCESSORS_ONLN);
  if (threads < 1) threads = 1;
  if (threads > B) threads = (int)B;
  job_t job;
  job.records = records; job.B = B; job.check_inputs = check_inputs;
  job.validity = validity; job.offsets = offsets; job.order = order;
  job.labels = labels; job.scores = scores; job.status = status;
  job.objective = objective;
  atomic_init(&job.next, 0);
  atomic_init(&job.error, 0);
  if (threads == 1) {
    worker(&job);
  } else {
    pthread_t* pool = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
    int started = 0;
    for (int k = 0; k < threads; ++k)
      if (pthread_create(&pool[k], NULL, worker, &job) == 0) ++started;
    if (started == 0) worker(&job);
    for (int k = 0; k < started; ++k) pthread_join(pool[k], NULL);
    free(pool);
  }
  free(offsets); free(order);
  return atomic_load(&job.error);
}

int ffa_oracle_emission_validity(const ffa_oracle_record* records, int64_t B,
                                 uint8_t* valid) {
  if (B <= 0 || !records || !valid) return -1;
  for (int64_t i = 0; i < B; ++i) {
    const float* v = records[i].emissions;
    const int64_t n = records[i].T * records[i].V;
    int ok = 1;
    /* NaN and +inf are invalid; -inf is allowed (alignment.cu:885-887). */
    for (int64_t k = 0; k < n; ++k)
      if (isnan(v[k]) || v[k] == INFINITY) { ok = 0; break; }
    valid[i] = (uint8_t)ok;
  }
  return 0;
}
