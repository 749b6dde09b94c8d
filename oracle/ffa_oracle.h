/*
 * ffa_oracle.h -- CPU restatement of the reference aligner's conventional
 * path.  TEST INFRASTRUCTURE ONLY: the product (fast_forced_aligner_b200)
 * never links, loads or calls this code.  Only tests/, the smoke() entry
 * point and bench.py's CPU baseline use it, as the checker.
 *
 * Parity anchors (reference = brthor/fast-forced-aligner):
 *   states / validation  src/fast_forced_aligner/csrc/alignment.cu:852-874
 *   DP init              alignment.cu:404-412
 *   DP recurrence        alignment.cu:414-429
 *   terminal / status    alignment.cu:496-510
 *   traceback / finish   alignment.cu:641-667
 *   emission validity    alignment.cu:879-891
 */
#ifndef FFA_ORACLE_H
#define FFA_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ffa_oracle_record {
  const float* emissions;   /* host, row-major [T, V] fp32 */
  const int64_t* targets;   /* host, [U] int64 (may be NULL when U == 0) */
  int64_t T;
  int64_t V;
  int64_t U;
  int64_t blank;
} ffa_oracle_record;

/* Status codes shared with the product (alignment.py:88-94). */
enum {
  FFA_ORACLE_OK = 0,
  FFA_ORACLE_NO_PATH = 1,
  FFA_ORACLE_MASKED = 2,
  FFA_ORACLE_BAD_TARGET = 3,
  FFA_ORACLE_TOO_FEW_FRAMES = 4
};

/*
 * Conventional max-plus Viterbi alignment of B independent records.
 * Outputs are packed in record order: labels/scores hold sum(T_i) entries.
 * validity may be NULL (no emission mask).  threads <= 0 means one thread
 * per online CPU.  Returns 0, or a negative value for malformed arguments
 * (including target IDs outside [0, V) when check_inputs == 0, which the
 * reference leaves undefined).
 */
int ffa_oracle_align(const ffa_oracle_record* records, int64_t B,
                     int check_inputs, const uint8_t* validity, int threads,
                     int64_t* labels, float* scores, int32_t* status,
                     float* objective);

/* 1 if a record holds no NaN and no +inf (alignment.cu:881-891), else 0. */
int ffa_oracle_emission_validity(const ffa_oracle_record* records, int64_t B,
                                 uint8_t* valid);

#ifdef __cplusplus
}
#endif
#endif
