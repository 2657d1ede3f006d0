/*
 * d3moe_selftest.h — test-only library libd3moe_selftest.so, built beside
 * libd3moe.so but not part of the product ABI.
 */
#ifndef D3MOE_SELFTEST_H_
#define D3MOE_SELFTEST_H_

#include "d3moe.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Self-test of the bounded-wait failure path of libd3moe.so: one thread waits,
 * through the same bounded wait every waiting kernel uses, on a barrier nothing
 * arrives on; after the wait limit (2 s) the kernel writes
 * D3_STATUS_WAIT_TIMEOUT to *status (device int32) and exits. No fault, and
 * the context stays usable. Returns D3_EINVAL for a null status word and
 * D3_ECUDA when the launch fails. No counterpart in the reference. */
D3_API int d3_wait_timeout_probe(int32_t* status, d3_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* D3MOE_SELFTEST_H_ */
