/*
 * CPU oracle for the streaming semi-CRF scan -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, loop-by-loop restatement of the reference implementation
 * (torch-semimarkov 0.2.0, src/torch_semimarkov/streaming/pytorch_reference.py,
 * nn.py:444-555 and helpers.py:365-544).  It is used by tests/ as the parity
 * checker and by bench.py as the CPU baseline ("port").  Nothing in the
 * torch_semimarkov_b200 package links or calls it.
 *
 * Parity of this restatement is pinned against golden vectors produced by the
 * reference itself (tests/golden/make_golden.py writes the .npz fixtures), see
 * tests/test_oracle_golden.py.
 *
 * Exported symbols (suffix _f64 = float64 oracle, _f32 = float32 baseline):
 *   oracle_checkpoint_interval, oracle_forward_*, oracle_backward_*,
 *   oracle_viterbi_*, oracle_score_gold_*.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

/* _compute_checkpoint_interval (pytorch_reference.py:25-45). */
int64_t oracle_checkpoint_interval(int64_t T, int64_t K) {
    int64_t opt = (int64_t)sqrt((double)(T * K));
    return opt > K ? opt : K;
}

int oracle_num_threads_available(void) {
#ifdef _OPENMP
    extern int omp_get_max_threads(void);
    return omp_get_max_threads();
#else
    return 1;
#endif
}

#define REAL double
#define SUFFIX f64
#define EXP exp
#define LOG log
#define NEG_INF_R (-1e9)
#include "semicrf_oracle_impl.h"
#undef REAL
#undef SUFFIX
#undef EXP
#undef LOG
#undef NEG_INF_R

#define REAL float
#define SUFFIX f32
#define EXP expf
#define LOG logf
#define NEG_INF_R (-1e9f)
#include "semicrf_oracle_impl.h"
#undef REAL
#undef SUFFIX
#undef EXP
#undef LOG
#undef NEG_INF_R
