/*
 * ref_threads.c -- test infrastructure only.  Linked into the oracle build
 * of the reference executor so that the CPU baseline can state and set the
 * BLAS thread count it ran with (the reference itself leaves this to the
 * OPENBLAS_NUM_THREADS environment variable).
 */
void scipy_openblas_set_num_threads(int n);
int scipy_openblas_get_num_threads(void);

void oracle_ref_set_threads(int n) { scipy_openblas_set_num_threads(n); }
int oracle_ref_get_threads(void) { return scipy_openblas_get_num_threads(); }
