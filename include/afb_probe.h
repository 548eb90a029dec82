/* Device-ceiling probes for the step kernel of libafb (measurement utility, no counterpart in the reference).
 *
 * The step kernel's cost is dominated by gathering, for every synapse of the light cone, one 512-byte
 * row of state (256 float16 positions) from L2 into the SM.  afb_probe_gather runs that access pattern
 * alone through one load path: n_rows rows of a slab, in the order given by `rows`, each row read as
 * 32 x 16 bytes and reduced to one word per warp so that no load can be dropped.
 * Bytes moved = n_rows * 512 (+ 4 per index).  Timing is the caller's (events around the call on `stream`).
 */
#ifndef AFB_PROBE_H
#define AFB_PROBE_H

#include <stdint.h>
#include <stddef.h>

#include "afb.h"

#ifdef __cplusplus
extern "C" {
#endif

#define AFB_PROBE_LDG 0            /* 16-byte global loads into registers, 8 in flight per lane */
#define AFB_PROBE_CPASYNC 1        /* cp.async (16 bytes per lane) into a shared-memory ring, 3 groups of 4 rows in flight per warp */
#define AFB_PROBE_CPASYNC_READ 2   /* the same, and every row read back from shared memory */
#define AFB_PROBE_TMA 3            /* tile::gather4 (4 rows per copy) into the ring, completion on mbarriers */
#define AFB_PROBE_TMA_READ 4       /* the same, and every row read back from shared memory */
#define AFB_PROBE_LDG4 5           /* as AFB_PROBE_LDG with 4 loads in flight per lane */
#define AFB_PROBE_LDG16 6          /* as AFB_PROBE_LDG with 16 loads in flight per lane */
#define AFB_PROBE_LDG_NARROW8 7    /* 256-byte rows (each slab row as two), 8 bytes per lane, 8 in flight */
#define AFB_PROBE_LDG_NARROW16 8   /* the same with 16 in flight */

/* Words the sink needs for a launch on the current device. */
AFB_API int64_t afb_probe_gather_sink_words(void);

/* path: AFB_PROBE_*; blocks_per_sm: CTAs of 256 threads per SM (1..8 on the register paths, 1..3 on the
 * ring paths; 0 = the maximum); slab: slab_rows x 512 bytes, 16-byte aligned; rows: n_rows int32 row
 * numbers (an index outside [0, slab_rows) reads row 0 on the ring paths and nothing on the register
 * paths; on the narrow paths the rows are 256 bytes and the range is [0, 2 slab_rows); the ring paths need
 * n_rows % 4 == 0); sink: afb_probe_gather_sink_words() words.
 * Returns AFB_OK or a negative code. */
AFB_API int afb_probe_gather(int path, int blocks_per_sm, const void *slab, int64_t slab_rows, const int32_t *rows,
                             int64_t n_rows, uint32_t *sink, int64_t sink_words, void *stream);

#ifdef __cplusplus
}
#endif

#endif
