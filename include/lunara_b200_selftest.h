/*
 * lunara_b200_selftest.h -- internal self-test entry points of liblunara_b200.so.
 *
 * These are not part of the kernel ABI in lunara_b200.h and have no
 * counterpart in the reference: they exist so that tests can check device
 * code paths that no product input reaches on purpose. Both return 0 on
 * success, 1 for bad arguments and 3 when the launch failed.
 */
#ifndef LUNARA_B200_SELFTEST_H
#define LUNARA_B200_SELFTEST_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* y[i] = 2^x[i] over n device floats by the FMA-pipe exponential: pair == 0
 * the scalar form, 1 the f32x2 form on pairs (both with MUFU ex2's range
 * behaviour: 0 below -126, NaN kept), 2 the clamped f32x2 form the attention
 * softmax runs (inputs below -126 give ~2^-126); n even when pair != 0.
 * Lets tests bound its error against exp2. */
int lunara_selftest_ex2_poly(const float* x, float* y, int64_t n, int pair, void* stream);

/* Launches one CTA that waits on an mbarrier nothing ever arrives on, with a
 * %globaltimer budget of budget_ns (1 us .. 1 s), exactly as the product
 * kernels bound every wait. When the budget runs out the kernel records
 * `site` (0x401 .. 0x4ff) in the device error word and returns; nothing
 * faults or hangs. Read the outcome with lunara_device_error(). */
int lunara_selftest_bounded_wait(uint64_t budget_ns, unsigned int site, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LUNARA_B200_SELFTEST_H */
