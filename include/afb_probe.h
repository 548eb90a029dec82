/* Gather-ceiling probe for the step kernel of libafb: a measurement utility in its own library
 * (alphafly_b200/libafb_probe.so, used by bench.py), not part of libafb.so.  It has no counterpart in the
 * reference.
 *
 * The step kernel's cost is dominated by gathering, for every synapse of the light cone, one 512-byte
 * row of state (256 float16 positions) from L2 into the SM.  afb_probe_gather runs that access pattern
 * alone through the step kernel's load path (16-byte loads into registers, 8 rows in flight per lane):
 * n_rows rows of a slab, in the order given by `rows`, each row read as 32 x 16 bytes and folded into one
 * word per warp so that no load can be dropped.  Bytes moved = n_rows * 512 (+ 4 per index).  Timing is
 * the caller's (events around the call on `stream`).
 */
#ifndef AFB_PROBE_H
#define AFB_PROBE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AFB_PROBE_OK 0
#define AFB_PROBE_EINVAL (-1)      /* a bad argument */
#define AFB_PROBE_ECUDA (-2)       /* a CUDA call failed */

#if defined(__GNUC__)
#define AFB_PROBE_API __attribute__((visibility("default")))
#else
#define AFB_PROBE_API
#endif

/* Words the sink needs for a launch on the current device. */
AFB_PROBE_API int64_t afb_probe_gather_sink_words(void);

/* blocks_per_sm: CTAs of 256 threads per SM, 1..8 (0 = 8, i.e. 64 warps per SM); slab: slab_rows x 512
 * bytes, 16-byte aligned; rows: n_rows int32 row numbers (an index outside [0, slab_rows) reads nothing);
 * sink: afb_probe_gather_sink_words() words.  Returns AFB_PROBE_OK or a negative code. */
AFB_PROBE_API int afb_probe_gather(int blocks_per_sm, const void *slab, int64_t slab_rows, const int32_t *rows,
                                   int64_t n_rows, uint32_t *sink, int64_t sink_words, void *stream);

#ifdef __cplusplus
}
#endif

#endif
