// Internal declarations shared by the kernel files and the C-ABI layer.
#pragma once
#include <utility>
#include <cuda_runtime.h>
#include <cstdint>

namespace fcqt {

struct FwdTab {            // analysis-engine tap table (one per use)
    const int* src;        // bin | conj << 16, or -1 for a zero tap
    const float* gain;     // window gain with all constants folded in
    const int2* seg;       // per band: first bin and length of its segment
};

struct InvTab {            // synthesis-engine tap table (one per use)
    const int* dest;       // plane * kPlaneStride + bin, or -1
    const float* gre;      // gain on the real part
    const float* gim;      // gain on the imaginary part
    const unsigned char* mask;  // per bin: bit p set when plane p holds a term
    // per quad n in [0, Q/2]: the masks of bins n, L - n, Q + n, Q - n in
    // bits 0-3, 4-7, 8-11, 12-15 (derived from `mask` at upload)
    const unsigned short* qmask;
    int nplanes;
};

constexpr int kMaxHostClasses = 8;   // block-length classes of the host tables
// internal classes: each host class splits into its octave bands and its
// side (per-tap table) bands, so a CTA holds one kind only
constexpr int kMaxClasses = 2 * kMaxHostClasses;
enum BandKind { kOctave = 0, kOctavePruned = 1, kSide = 2 };

struct BandSched {         // CTA ranges of the block-length classes for one launch
    int ncls;
    int M[kMaxClasses];
    int nb[kMaxClasses];       // bands in the class
    int first[kMaxClasses];    // first entry of the class in band_list
    int cta0[kMaxClasses + 1]; // first CTA of each class, cta0[ncls] = grid
    int kind[kMaxClasses];     // BandKind of the class
    int batch;
    float inv_batch;           // 1 / batch, for the instance -> (band, slice) split
};

constexpr int kMaxBands = 512;
constexpr int kInlineBands = 160;
constexpr int kMaxGroups = 16;

// Coefficient layout of the sliced transform: one interleaved complex buffer
// holding, group after group, blocks [rows][b][S * M] (octave groups: slice
// coefficients in time order, each slice's block rolled by +M/4 (even slice)
// or -M/4 (odd slice), sliced.py:119-146) and [rows][S][M] (DC and Nyquist
// side groups, not rolled).  S == 0 selects the per-slice heap layout.
struct SliceLayout {
    int S;                          // slices per signal row in this call
    int slice0;                     // global index of the first slice (roll parity)
    long long goff[kMaxGroups];     // complex offset of each group block
    int grows[kMaxGroups];          // bands in the group
    int groll[kMaxGroups];          // 1: coefficients rolled by +-M/4
};

// where a slice's samples come from (analysis front end) or go to
// (synthesis back end).  S == 0: contiguous [B][65536] slices.  S > 0:
// local slice s is global slice g = slice0 + s of a [rows][length] signal and
// covers global samples 2H (g - 1) + j, j < 4H (H = 16384), in the quarter-
// rolled order of sliced.py:106-117 (sample n of the slice is
// j = (n +- H) mod 4H, + for even g); the window (if not null) multiplies
// sample j.  The buffer row holds global samples [sample0, sample0 + count)
// at stride ld; samples outside that window or outside [0, length) read as
// zero / are dropped.  Outputs overlap-add (two slices per sample) into a
// zeroed buffer.
struct SigMap {
    const float* x;        // input signal (analysis engine)
    float* y;              // output signal (synthesis engine)
    long long ld;          // row stride in floats
    long long length;      // global signal length
    long long sample0;     // global sample index of buffer column 0
    long long count;       // samples held per buffer row
    int S;
    int slice0;
    const float* window;   // [65536] or null
    // squared-error mode of the contiguous layout (S == 0), for an MSE loss:
    // the analysis engine reads s * (x - target) with s = scale (times
    // *scale_dev when not null); the synthesis engine stores y and writes one
    // partial sum of (y - target)^2 per CTA into partial[CTA]
    const float* target;
    const float* scale_dev;
    float scale;
    float* partial;
};

// input / output mode of the spectrum kernels
enum SigMode { kSigPlain = 0, kSigSliced = 1, kSigSqErr = 2 };

// everything a band kernel needs besides the per-tap tables, passed by value
// (kernel parameters live in the constant bank: no dependent global loads)
struct BandParams {
    BandSched sc;
    const float2* tw2048;  // W_2048^e, forward sign
    const float2* twrows;  // per-block-length twiddle slots (band_twiddle_rows)
    int ncoef;
    // per band in class order: {heap offset, lo (octave) | band id (side),
    // l | Lg << 16, flags: bit 0 side band, bits 4-7 synthesis plane, bits
    // 8-11 adjoint plane, bits 12-15 group, bits 16-23 row in group}.  The
    // descriptors of a bank of at most kInlineBands bands ride in the kernel
    // parameters (constant bank, no dependent global load before a CTA's
    // first copy); larger banks run a kernel instantiation that reads them
    // from device memory (desc).  2.5 KB of parameters rather than 8 KB keeps
    // eager launches cheap.
    int4 desc_inline[kInlineBands];
    const int4* desc;
    int ext;               // more than kInlineBands bands: read desc
    SliceLayout sl;
    // wait-status word in the caller's workspace header (null: none); a
    // bounded wait that gives up adds 1 to it
    unsigned* status;
    // test hook (cqt_debug_expire_waits): the staging barrier expects 16
    // bytes that no copy delivers, so every bounded wait runs out
    int expire_waits;
    int stride;            // complex values per spectrum row / colour plane
};

struct CoefPtr {           // coefficient heap addressing
    float* re;             // planar: real plane; interleaved: complex base
    float* im;             // planar: imaginary plane; interleaved: unused
    int interleaved;       // 0 planar [B, ncoef] x 2, 1 complex [B, ncoef]
};

// points held in registers per band-kernel thread (16 or 32); the band
// schedules in bands.cu follow it
#ifndef FCQT_BAND_P
#define FCQT_BAND_P 16
#endif
constexpr int kBandP = FCQT_BAND_P;
// 128 threads of 16 points: 2048 points per band CTA, eight CTAs per SM (the
// fastest of 128 / 256 / 512 measured; 128 is the least a 2048-point band needs)
#ifndef FCQT_BAND_THREADS
#define FCQT_BAND_THREADS 128
#endif
constexpr int kBandThreads = FCQT_BAND_THREADS;
constexpr int kBandCap = kBandThreads * kBandP;   // points per band CTA

BandSched make_sched(int ncls, const int* M, const int* nb, const int* first, const int* kind,
                     int batch);

cudaError_t init_kernel_attributes();
struct SpecTables {        // packed-spectrum engine twiddles (device)
    const float2* hi;      // W_65536^(256 e), e < 256
    const float2* lo;      // W_65536^e, e < 256
    const float2* rows;    // per-stage twiddle rows (spectrum_twiddle_rows)
    int nslice;            // samples per slice: 65536 or 32768
};

// ---------------------------------------------------------------------------
// Programmatic dependent launch: every kernel lets the next kernel of its
// stream launch once all of its own CTAs have started (pdl_launch_dependents
// at entry); the next kernel's CTAs run their prologue on the SMs the tail
// frees and execute pdl_wait -- which returns only when the previous grid
// has completed and its memory is visible -- before they read or write any
// buffer another kernel touches.  Without the launch attribute both are no-ops.
#ifndef FCQT_PDL
#define FCQT_PDL 1
#endif

__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
}

// PDL pays where launch and tail are a large share of a kernel: batches of
// at most kPdlMaxBatch slices (measured: -7 % at one slice, -4 % at 64, +1 %
// at 1024, where the early CTAs only sit waiting)
constexpr int kPdlMaxBatch = 128;

template <class... KArgs, class... Args>
cudaError_t launch_pdl(bool pdl, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = (FCQT_PDL && pdl) ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

int spectrum_twiddle_count();
void spectrum_twiddle_rows(float2* out);   // host, double precision

cudaError_t launch_spectrum_fwd(const SigMap& in, float2* X, const SpecTables& st, int batch,
                                cudaStream_t s);
cudaError_t launch_spectrum_inv(const float2* E, const InvTab& tab, const SigMap& out,
                                const SpecTables& st, int batch, cudaStream_t s);
// CTAs of one spectrum launch over `batch` slices (partial sums of the
// squared-error mode: one per CTA)
inline int spectrum_ctas(int batch) { return 2 * batch; }
// loss = scale * sum of the n partials, in a fixed order (one CTA)
cudaError_t launch_sqerr_finish(const float* partial, int n, float scale, float* loss,
                                cudaStream_t s);
cudaError_t read_wait_timeouts(unsigned* count);   // expired bounded waits (device)

// overlap-add halo over peer memory (halo.cu)
struct HaloDev;
struct HaloState {
    int device;
    int rows;
    long long hop;
    char* own;          // own exchange buffer (cudaMalloc, IPC-exported)
    char* left;         // left neighbour's buffer (IPC-mapped) or null
    char* right;        // right neighbour's buffer (IPC-mapped) or null
    HaloDev* dv;        // status word, CTA counters, failed epochs (own memory)
    unsigned long long wait_ns;   // bound of every wait on a neighbour
};
cudaError_t halo_create(HaloState* h, void* handle_out);
cudaError_t halo_open(const void* handle, char** out);
cudaError_t halo_send(HaloState* h, const float* src, long long ld, long long epoch,
                      cudaStream_t s);
cudaError_t halo_recv_add(HaloState* h, float* dst, long long ld, long long epoch,
                          cudaStream_t s);
cudaError_t halo_status(HaloState* h, unsigned* expired, int clear);
void halo_destroy(HaloState* h);
cudaError_t launch_bands_fwd(const float2* X, const FwdTab& tab, const BandParams& bp,
                             CoefPtr out, cudaStream_t s);
cudaError_t launch_bands_inv(CoefPtr in, const InvTab& tab, int which, const BandParams& bp,
                             float2* E, cudaStream_t s);
// the band kernels' twiddle slots, one per block length 16..2048, built on
// the host from the W_2048 table (float2 count, then the rows)
int band_twiddle_count();
void band_twiddle_rows(float2* out, const float2* w2048);

}  // namespace fcqt
