/*
 * gdn_testing.h -- test hooks of libgdn_b200.so.  They have no counterpart
 * in the reference and are not part of the operator's interface: they exist
 * so that a test can drive the chunked kernels' bounded-wait error path
 * without faulting or hanging the GPU.
 *
 * Every tcgen05/TMA pipeline wait in the chunked prefill kernels gives up
 * after a time limit (2 s by default), records GDN_ETIMEOUT for
 * gdn_check_device_errors, drains its own copies and MMAs, frees its tensor
 * memory and returns.  A test shortens the limit, injects a fault that leaves
 * one wait unsatisfied (a barrier that nothing completes), checks that
 * gdn_check_device_errors reports GDN_ETIMEOUT, then restores both settings
 * and checks that a normal call still gives correct results.
 *
 * Both settings are per device (the current one) and apply to kernels
 * launched after the call; do not change them while chunked work is in
 * flight.
 */
#ifndef GDN_TESTING_H
#define GDN_TESTING_H

#include <stdint.h>

#include "gdn_api.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Wait limit of the chunked kernels in nanoseconds; 0 restores the 2 s
 * default. */
gdn_status gdn_test_set_wait_limit(uint64_t ns);

/* Injected fault: 0 = none; 1 = the chunked scan's loader never issues the
 * V tile of each sequence's first chunk, so the stages waiting for it time
 * out. */
gdn_status gdn_test_inject_fault(int32_t fault);

#ifdef __cplusplus
}
#endif

#endif /* GDN_TESTING_H */
