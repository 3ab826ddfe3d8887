/* mxfp8_checked.h -- the checked build of the library, libmxfp8_checked.so.
 *
 * Same sources and C ABI as libmxfp8.so (include/mxfp8.h), compiled with
 * MXFP8_CHECKED: every global store of every kernel is tested against the
 * bytes of the output it belongs to (Q rows [q, q + (q_rows-1)*ld_q + q_cols),
 * the packed scale storage, the dequantized output) and against its own
 * alignment.  A store that fails the test is skipped and sets bit 16 of the
 * device status word (mxfp8_device_status); nothing traps.  It exists to run
 * the test suite's layout battery where no memory checker may run, and is not
 * meant for production (every store pays the test).
 *
 * No counterpart in the reference (it has no sanitizer or checked build). */
#ifndef MXFP8_CHECKED_H
#define MXFP8_CHECKED_H

#include "mxfp8.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Narrow every later call's output windows by `bytes` (0 .. 2^20; 0 = the
 * exact outputs), so that a test can see the guards skip the stores at the
 * end of each output and report them.  Process-wide; the skipped stores would
 * have gone to the caller's own buffers. */
MXFP8_API int mxfp8_checked_window_slack(int64_t bytes);

#ifdef __cplusplus
}
#endif

#endif /* MXFP8_CHECKED_H */
