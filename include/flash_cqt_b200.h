/* flash_cqt_b200.h -- C ABI of the B200 (sm_100a) constant-Q transform engines.
 *
 * The reference (Flash-CQT) binds its CUDA code through pybind11 functions that
 * take torch tensors (flash_cqt/csrc/packedfft.cu:256-262, radix.cu:116-121)
 * and are JIT-built on first use (flash_cqt/fused.py:39-146).  This library
 * replaces that boundary with plain pointers, sizes and a CUDA stream:
 *
 *   reference entry point(s)                          replaced by
 *   -----------------------------------------------   ----------------------
 *   FusedOctCQT.__init__ table build + .to(dev)       cqt_tables_upload
 *     (fused.py:229-476, trainable.py:39-61)
 *   trainable.py:75-89   _analysis  = pack + fft3     cqt_analysis
 *     (packedfft.cu:100-126) + fwd_bands (radix.cu:46-62)
 *   trainable.py:100-109 _synthesis = zero + inv_bands cqt_synthesis
 *     (radix.cu:64-91) + inv_tail (packedfft.cu:233-254)
 *   trainable.py:111-122 _adj_analysis = adj_bands    cqt_adj_analysis
 *     (radix.cu:93-114) + inv_tail
 *   trainable.py:124-139 _adj_synthesis = fft3 +      cqt_adj_synthesis
 *     fwd_bands with the route_b table
 *   FusedOctCQT._workspace (fused.py:517-523)         cqt_workspace_bytes
 *
 * Conventions
 *   - Every pointer except the host tables of cqt_tables_upload is a device
 *     pointer on the device the tables were uploaded to; that device must be
 *     current when an entry point is called.
 *   - x, y, gx, gy: float32 [batch][slice_len] (65536, or 32768 for tables
 *     built for 32768-sample slices), 8-byte aligned (CQT_ERR_ARG otherwise;
 *     rows at 16-byte alignment take the vector store path).
 *   - coefficients: the heap of one slice is ncoef complex values (octave
 *     groups lowest first, then the DC and the Nyquist side block, each group
 *     [bins][M] row-major).  layout CQT_LAYOUT_PLANAR: c_re and c_im are two
 *     float32 [batch][ncoef] arrays; CQT_LAYOUT_COMPLEX: c_re is an interleaved
 *     complex64 [batch][ncoef] array and c_im is ignored (may be NULL).
 *   - workspace: caller-owned device scratch of at least
 *     cqt_workspace_bytes(t, batch) bytes, 16-byte aligned; it may be reused
 *     between calls that are ordered on one stream.  Its first 256 bytes are a
 *     header holding the wait-status word (cqt_workspace_waits): zero them
 *     once when the workspace is allocated.
 *   - One call takes fewer than 2^24 / (largest number of bands sharing one
 *     block length) slices (batch, or rows x slices); 349,525 for the default
 *     bank, far more than fit in device memory.  Larger calls return
 *     CQT_ERR_ARG.
 *   - All entry points are asynchronous on `stream` (a cudaStream_t, NULL =
 *     legacy default stream), allocate nothing, never synchronise, and may be
 *     captured into a CUDA graph.  One cqt_tables may serve several streams.
 *   - Return value: CQT_OK or a negative error code; cqt_last_error() gives a
 *     message for the calling thread.
 */
#ifndef FLASH_CQT_B200_H
#define FLASH_CQT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CQT_OK 0
#define CQT_ERR_ARG (-1)    /* bad argument (null pointer, size, layout) */
#define CQT_ERR_CUDA (-2)   /* CUDA runtime error (launch, allocation, copy) */
#define CQT_ERR_DEVICE (-3) /* wrong current device or no device */

#define CQT_LAYOUT_PLANAR 0
#define CQT_LAYOUT_COMPLEX 1

#define CQT_SLICE 65536   /* default slice length; 32768 is the other one built */

/* Host-side tables, built once per filterbank (the Python side builds them in
 * float64 and rounds once).  Per-tap arrays have ncoef entries in heap order. */
typedef struct cqt_host_tables {
    int32_t nbands;             /* <= 512 */
    int32_t ncoef;
    const int32_t* band_off;    /* [nbands] heap offset of each band */
    const int32_t* band_list;   /* [nbands] band ids grouped by class */
    /* [nbands][4] geometry {lo, l, Lg, flags}: an octave band's tap m maps to
     * bin lo + ((m + l) mod M) when (m + l) mod M < Lg; flags bit 0 marks the
     * side (DC / Nyquist) bands that use the per-tap tables instead, bits 4-7
     * and 8-11 hold the colour plane of the band for synthesis and for the
     * transpose of the analysis.  Upload checks it against the per-tap tables. */
    const int32_t* band_geom;
    /* coefficient groups in heap order (octave groups, then the DC and the
     * Nyquist side groups): bands per group and whether the sliced layout
     * rolls the group's blocks by +-M/4 (1 for octave groups, 0 for sides) */
    int32_t ngroups;            /* <= 16 */
    const int32_t* group_count;
    const int32_t* group_roll;
    int32_t nclasses;           /* <= 8 block-length classes, largest first */
    const int32_t* class_len;   /* [nclasses] block length M (32..2048) */
    const int32_t* class_count; /* [nclasses] bands in the class */
    const int32_t* class_first; /* [nclasses] first class entry in band_list */
    /* analysis-engine tap tables: src = bin | conj << 16, or -1; seg =
     * [nbands][2] (first bin, bin count) of the contiguous half-spectrum
     * segment that holds every live tap of the band (count <= M) */
    const int32_t* an_src;  const float* an_gain;   /* analysis */
    const int32_t* an_seg;
    const int32_t* as_src;  const float* as_gain;   /* transpose of synthesis */
    const int32_t* as_seg;
    /* synthesis-engine tap tables: dest = plane * 32776 + bin, or -1 */
    const int32_t* sy_dest; const float* sy_gre; const float* sy_gim;
    const uint8_t* sy_mask; int32_t sy_nplanes;     /* synthesis */
    const int32_t* aa_dest; const float* aa_gre; const float* aa_gim;
    const uint8_t* aa_mask; int32_t aa_nplanes;     /* transpose of analysis */
    const float* tw2048;        /* [2048][2] W_2048^e */
    const float* tw_hi;         /* [256][2]  W_65536^(256 e) */
    const float* tw_lo;         /* [256][2]  W_65536^e */
    /* samples per slice: 65536 or 32768 (0 means 65536).  The bins of the
     * per-tap tables run to slice_len / 2, and plane slots and masks use the
     * stride slice_len / 2 + 8 (32776 or 16392). */
    int32_t slice_len;
} cqt_host_tables;

typedef struct cqt_tables cqt_tables; /* device-resident tables (opaque) */

/* Copy the tables to `device` (cudaMalloc + cudaMemcpy, done once). */
int cqt_tables_upload(const cqt_host_tables* host, int device, cqt_tables** out);
int cqt_tables_free(cqt_tables* t);
int32_t cqt_ncoef(const cqt_tables* t);
int32_t cqt_slice_len(const cqt_tables* t);   /* 65536 or 32768 */

/* Scratch bytes needed by any entry point at this batch size. */
size_t cqt_workspace_bytes(const cqt_tables* t, int batch);

/* x [batch][65536] -> coefficient heap (OctCQT.fwd, oct_cqt.py:84-96). */
int cqt_analysis(const cqt_tables* t, const float* x, float* c_re, float* c_im,
                 int layout, int batch, void* workspace, size_t workspace_bytes,
                 void* stream);

/* coefficient heap -> y [batch][65536] (OctCQT.bwd, oct_cqt.py:98-117). */
int cqt_synthesis(const cqt_tables* t, const float* c_re, const float* c_im,
                  int layout, float* y, int batch, void* workspace,
                  size_t workspace_bytes, void* stream);

/* transpose of the analysis: coefficient gradients (dL/dRe, dL/dIm) -> dL/dx. */
int cqt_adj_analysis(const cqt_tables* t, const float* g_re, const float* g_im,
                     int layout, float* gx, int batch, void* workspace,
                     size_t workspace_bytes, void* stream);

/* transpose of the synthesis: dL/dy -> coefficient gradients. */
int cqt_adj_synthesis(const cqt_tables* t, const float* gy, float* g_re,
                      float* g_im, int layout, int batch, void* workspace,
                      size_t workspace_bytes, void* stream);

/* MSE training loss folded into the engines (the optional fused MSE of the
 * adjoint-synthesis entry point; the reference runs the loss and its
 * gradient as separate torch operations between its engines, the train step
 * of bench/profile_step.py and trainable.py:180-191).
 *
 * cqt_synthesis_sqerr: y = synthesis(coefficients) exactly as cqt_synthesis,
 * and *loss (one device float) = loss_scale * sum over all batch * 65536
 * samples of (y - target)^2, summed in a fixed order (deterministic; the
 * mean is loss_scale = 1 / (batch * 65536)).  target as y (8-byte aligned).
 * An empty batch writes 0.
 *
 * cqt_adj_synthesis_sqerr: the transpose of the synthesis (as
 * cqt_adj_synthesis) applied to dL/dy = s * (y - target), formed while the
 * signal is loaded, with s = scale * (*scale_dev) (scale_dev: an optional
 * device float such as the loss gradient dL/dloss; NULL means 1).  For the
 * mean squared error, scale = 2 / (batch * 65536). */
int cqt_synthesis_sqerr(const cqt_tables* t, const float* c_re, const float* c_im,
                        int layout, float* y, const float* target, float* loss,
                        float loss_scale, int batch, void* workspace,
                        size_t workspace_bytes, void* stream);
int cqt_adj_synthesis_sqerr(const cqt_tables* t, const float* y, const float* target,
                            float scale, const float* scale_dev, float* g_re,
                            float* g_im, int layout, int batch, void* workspace,
                            size_t workspace_bytes, void* stream);

/* Diagnostic: launch one kernel of the pipeline on its own, for per-kernel
 * timing and profiling.  stage: 0 spectrum_fwd (in = signal, out = workspace
 * spectrum), 1 bands_fwd analysis (in = workspace spectrum, out = coefficients
 * c_re/c_im), 2 bands_inv synthesis (in = coefficients, out = workspace
 * planes), 3 spectrum_inv synthesis (in = workspace planes, out = signal).
 * Stages 1 and 3 read what stages 0 and 2 left in the workspace. */
#define CQT_STAGE_SPECTRUM_FWD 0
#define CQT_STAGE_BANDS_FWD 1
#define CQT_STAGE_BANDS_INV 2
#define CQT_STAGE_SPECTRUM_INV 3
int cqt_launch_stage(const cqt_tables* t, int stage, const float* sig_in,
                     float* sig_out, float* c_re, float* c_im, int layout,
                     int batch, void* workspace, size_t workspace_bytes,
                     void* stream);

/* cqt_analysis without a workspace argument, for callers that cannot
 * allocate device memory (e.g. a real-time audio callback, where cudaMalloc
 * may block and synchronise the device).  No counterpart in the reference.
 * Scratch comes from a static device array inside this library sized for at
 * most 8 slices (batch > 8 returns CQT_ERR_ARG); every GPU that loads the
 * library holds those 2 MiB until exit.  The first call on a device (that
 * device current) looks the array up with cudaGetSymbolAddress, which may
 * make the CUDA runtime load this library's device code and so allocate and
 * synchronise: make one warm-up call per device at start-up, off the
 * real-time thread and before any stream capture (batch 0 suffices).  After
 * it, calls allocate nothing and never synchronise.  All calls share the
 * array: calls that overlap on the GPU race. */
int cqt_analysis_noalloc(const cqt_tables* t, const float* x, float* c_re,
                         float* c_im, int layout, int batch, void* stream);

/* ---- Sliced streaming transform (SlicedCQT, sliced.py:41-167) ----------
 * A signal of `rows` rows and global length `length` is cut into
 * S = cqt_sliced_count(length) slices of 65536 samples at 50 % overlap:
 * global slice g covers global samples 32768 (g - 1) + j, j < 65536,
 * multiplied by the slice window (analysis), and is quarter-rolled (-16384
 * for even g, +16384 for odd g).  One call processes slices
 * [slice0, slice0 + slices) of every row, so a long stream can be split
 * into slice ranges (e.g. one per GPU).
 * Signal buffers (cqt_signal) hold, per row at stride ld, the global samples
 * [sample0, sample0 + count); samples outside that window or outside
 * [0, length) read as zero (inputs) or are dropped (outputs).  Outputs are
 * zeroed, then overlap-added: a sample gets the terms of the (at most two)
 * slices of the call that cover it, order-independent (deterministic).
 * Coefficients live in one interleaved complex64 buffer of
 * rows * slices * ncoef values, group after group (group k at offset
 * rows * slices * sum_{k' < k} count_k' M_k'): octave groups as
 * [rows][count][slices * M] (slices in time order, each slice's block rolled
 * by +M/4 (even g) or -M/4 (odd g)), side groups as [rows][slices][M] --
 * exactly the blocks of SlicedCQT.fwd.  Workspace:
 * cqt_workspace_bytes(t, rows * slices). */
typedef struct cqt_signal {
    float* data;        /* device; const for inputs */
    int64_t ld;         /* row stride in floats, >= count */
    int64_t sample0;    /* global sample held in data[0] (may be negative) */
    int64_t count;      /* samples held per row */
    int64_t length;     /* global signal length */
} cqt_signal;

typedef struct cqt_slices {
    int32_t rows;
    int32_t slice0;          /* global index of the first slice of the call */
    int32_t slices;          /* slices per row in the call */
    const float* window;     /* device float32[65536] slice window; analysis
                                and its transpose only */
} cqt_slices;

/* slices of a stream of `length` samples at 65536-sample slices; for
 * 32768-sample slices the same formula with a hop of 16384:
 * (ceil(length / (slice_len / 4)) + 1) / 2 + 1 */
int cqt_sliced_count(int64_t length);
int cqt_sliced_analysis(const cqt_tables* t, const cqt_signal* x, const cqt_slices* sl,
                        float* coef, void* workspace, size_t workspace_bytes, void* stream);
int cqt_sliced_synthesis(const cqt_tables* t, const float* coef, const cqt_slices* sl,
                         const cqt_signal* y, void* workspace, size_t workspace_bytes,
                         void* stream);
/* transposes: coefficient gradients -> dL/dx (window applied, overlap-add),
 * dL/dy -> coefficient gradients (no window) */
int cqt_sliced_adj_analysis(const cqt_tables* t, const float* gcoef, const cqt_slices* sl,
                            const cqt_signal* gx, void* workspace, size_t workspace_bytes,
                            void* stream);
int cqt_sliced_adj_synthesis(const cqt_tables* t, const cqt_signal* gy, const cqt_slices* sl,
                             float* gcoef, void* workspace, size_t workspace_bytes,
                             void* stream);

/* Diagnostic (no reference counterpart): the number of bounded waits in the
 * kernels (TMA bulk-copy completions) that gave up on the current device since
 * the library was loaded.  Every wait polls a fixed number of times and then
 * counts itself here and lets the kernel finish instead of hanging; a nonzero
 * count means results computed since then are not trustworthy.  Synchronous
 * (reads device memory). */
int cqt_wait_timeouts(unsigned int* count);

/* ---- Overlap-add halo over peer memory (no reference counterpart: the
 * reference is single-GPU) -----------------------------------------------
 * A long stream's slices range-partitioned over ranks (one process per GPU)
 * overlap-add locally; rank r > 0 sends the first hop of its output window
 * (rows x hop floats) to rank r - 1, which adds it into its last owned hop.
 * Each rank creates one exchange (a receive buffer exported by CUDA IPC,
 * handle of CQT_HALO_HANDLE_BYTES), learns its neighbours' handles by any
 * host means (e.g. an all-gather), and connects.  Calls are stream-ordered
 * and take an epoch, 1, 2, ... per exchange: send stores the hop into the
 * left neighbour's buffer with plain peer stores once that neighbour has
 * consumed epoch - 1, then raises its flag; recv_add waits for its own flag
 * to reach the epoch, adds, and acknowledges.  Every wait is bounded (10 s
 * by default) and a wait that gives up is counted in cqt_halo_waits (the data movement is
 * skipped); nothing hangs.  No multicast or switch reduction is used. */
#define CQT_HALO_HANDLE_BYTES 64
typedef struct cqt_halo cqt_halo;
/* rows: 1..65535 signal rows; wait_ms: the bound of every wait on a
 * neighbour (0: 10 s) */
int cqt_halo_create(int device, int rows, int64_t hop, int wait_ms, cqt_halo** out,
                    void* handle);
int cqt_halo_connect(cqt_halo* h, const void* left_handle, const void* right_handle);
int cqt_halo_send(cqt_halo* h, const float* src, int64_t ld, int64_t epoch, void* stream);
int cqt_halo_recv_add(cqt_halo* h, float* dst, int64_t ld, int64_t epoch, void* stream);
int cqt_halo_waits(cqt_halo* h, unsigned int* expired, int clear);
int cqt_halo_free(cqt_halo* h);

/* Diagnostic (no reference counterpart): the bounded waits that gave up in
 * the calls that used `workspace` since its header was last cleared -- the
 * per-workspace, so per-call when checked after each call, form of
 * cqt_wait_timeouts.  Every band kernel of a call adds its expired waits to
 * the status word in the workspace header; a nonzero count means those
 * calls' results are not trustworthy.  Synchronous (reads, and with
 * clear != 0 zeroes, 4 bytes of device memory on the legacy default
 * stream). */
int cqt_workspace_waits(void* workspace, size_t workspace_bytes, unsigned int* expired,
                        int clear);

/* Test hook for the failure detection above (no reference counterpart):
 * while on != 0, every launch made by this process arms the band kernels'
 * staging barriers for 16 bytes more than their copies deliver, so every
 * bounded wait runs out (after 1 s) and is recorded; results are garbage.
 * Nothing faults or hangs; the context stays usable. */
int cqt_debug_expire_waits(int on);

/* Message of the last failed call on this thread ("" if none). */
const char* cqt_last_error(void);

/* ABI version of this header (major * 100 + minor). */
int cqt_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FLASH_CQT_B200_H */
