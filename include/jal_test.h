/*
 * jal_test.h -- test hooks of the C ABI: failure detection without a fault.
 *
 * No counterpart in the reference.  Every wait of the device code on a copy
 * or on another GPU is bounded; when one gives up, the kernel sets a bit of
 * the context's error word and runs to its end, and the host call returns
 * JAL_ERR_TIMEOUT with the position unchanged.  These entry points make one
 * such wait run out on purpose -- an mbarrier that expects more bytes than
 * are sent, an exchange word whose flag never matches -- so a test can check
 * that path on a GPU without faulting, trapping or hanging it.
 */
#ifndef JAL_TEST_H
#define JAL_TEST_H

#include <stddef.h>
#include <stdint.h>

#include "jal.h"

#ifdef __cplusplus
extern "C" {
#endif

/* From the next decode step on, the decode attention's last V-stage barrier
 * (in every output CTA) expects extra_bytes more than the copy sends, and
 * each copy wait gives up after wait_ns (0 = the default 2 s); extra_bytes =
 * 0 and wait_ns = 0 restore normal operation.  Contexts of the FAST numerics
 * on one GPU only (JAL_ERR_CAPABILITY_MISMATCH otherwise). */
int jal_context_test_stall_kv_copy(jal_context *ctx, uint32_t extra_bytes,
                                   uint64_t wait_ns);

/* Runs one RMSNorm-input decode GEMV of `mat` (Q4_0 / Q8_0, at most 8192
 * columns) whose input is a tensor-parallel exchange slot of one rank whose
 * words carry a flag that never matches, with a wait bound of wait_ns, and
 * reports how the device error word came back: JAL_ERR_TIMEOUT when the
 * exchange wait gave up (the expected outcome), JAL_OK when it did not.
 * elapsed_ms (may be NULL) receives the host-measured duration. */
int jal_test_peer_exchange_timeout(const jal_cached_matrix *mat, uint64_t wait_ns,
                                   double *elapsed_ms);

/* Step trace (a diagnostic, not a failure hook): decodes two greedy steps
 * from `token` at the current position (the position advances by two) with
 * the FAST single-GPU step captured in a graph whose reference-order kernels
 * stamp the globaltimer; the second (warm) step's stamps land in out, 8 per
 * launch: out[8 i] = launch i's first CTA start, out[8 i + 1] = its last
 * warp's end, out[8 i + 2 + k] = the latest time any of its CTAs reached
 * phase k (0 = not recorded; the attention kernels mark the grid-dependency
 * wait, their phase boundaries and their chains).  Launches that record
 * nothing (the embedding, the argmax) read all ones / 0.  *n_launches receives
 * the step's launch count; out_len (elements) bounds what is copied.  The
 * normal step graph is recaptured afterwards. */
int jal_context_trace_decode_step(jal_context *ctx, uint32_t token, uint64_t *out,
                                  size_t out_len, size_t *n_launches);

#ifdef __cplusplus
}
#endif
#endif /* JAL_TEST_H */
