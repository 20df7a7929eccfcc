// C ABI (include/flash_cqt_b200.h): table upload and the four stream-ordered
// entry points.  Each entry point validates its arguments, launches two
// kernels on the caller's stream and reports launch errors; none allocates
// or synchronises.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/flash_cqt_b200.h"
#include "engine.cuh"
#include "internal.h"

namespace fcqt {
cudaError_t init_spectrum_attributes();
cudaError_t init_band_attributes();
}  // namespace fcqt

using namespace fcqt;

struct cqt_tables {
    int device;
    int ncoef;
    int nbands;
    int ncls;   // internal classes (see BandKind)
    int cls_M[kMaxClasses], cls_nb[kMaxClasses], cls_first[kMaxClasses], cls_kind[kMaxClasses];
    FwdTab fwd[2];   // 0 analysis, 1 transpose of synthesis
    InvTab inv[2];   // 0 synthesis, 1 transpose of analysis
    const float2* tw2048;
    const float2* twrows;   // band twiddle slots
    const int4* desc;       // device copy in the blob, class order, see BandParams
    int4 desc_host[kInlineBands];   // the inline head of the same array
    int ngroups;
    int group_count[kMaxGroups], group_len[kMaxGroups], group_roll[kMaxGroups];
    SpecTables spec;
    int max_planes;
    int nslice, half, quarter, stride;   // slice geometry (65536 or 32768 samples)
    void* blob;
};

namespace {

thread_local std::string g_err;

int fail(int code, const char* msg) {
    g_err = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char* where) {
    char buf[512];
    std::snprintf(buf, sizeof buf, "%s: %s", where, cudaGetErrorString(e));
    g_err = buf;
    return CQT_ERR_CUDA;
}

int check_device(const cqt_tables* t) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev != t->device) {
        char buf[160];
        std::snprintf(buf, sizeof buf,
                      "tables live on device %d but device %d is current", t->device, dev);
        g_err = buf;
        return CQT_ERR_DEVICE;
    }
    return CQT_OK;
}

// workspace: a 256-byte header (the wait-status word, cqt_workspace_waits),
// the spectrum rows / colour planes, then the per-CTA partial sums of the
// squared-error entry points (16-byte aligned: the planes are)
constexpr size_t kWsHeader = 256;
size_t ws_planes(const cqt_tables* t, int batch) {
    return (size_t)batch * (size_t)t->max_planes * (size_t)t->stride * sizeof(float2);
}
size_t ws_need(const cqt_tables* t, int batch) {
    const size_t partials = ((size_t)spectrum_ctas(batch) * sizeof(float) + 15) & ~(size_t)15;
    return kWsHeader + ws_planes(t, batch) + partials;
}
float* ws_partials(const cqt_tables* t, int batch, void* ws) {
    return reinterpret_cast<float*>(static_cast<char*>(ws) + kWsHeader + ws_planes(t, batch));
}

// what one call's kernels use: the spectrum rows / planes and the status word
struct Scratch {
    float2* rows;
    unsigned* status;
};
Scratch scratch_of(void* ws) {
    return Scratch{reinterpret_cast<float2*>(static_cast<char*>(ws) + kWsHeader),
                   static_cast<unsigned*>(ws)};
}

std::atomic<int> g_expire_waits{0};   // cqt_debug_expire_waits

// the band kernels split an instance index into (band, slice) with a float
// reciprocal, exact while slices x (bands of one block length) < 2^24
int check_slices(const cqt_tables* t, long long slices) {
    int mx = 1;
    for (int c = 0; c < t->ncls; ++c) mx = t->cls_nb[c] > mx ? t->cls_nb[c] : mx;
    if (slices * mx >= (1LL << 24))
        return fail(CQT_ERR_ARG, "too many slices in one call (split the batch)");
    return CQT_OK;
}

int check_common(const cqt_tables* t, int batch, void* ws, size_t ws_bytes, int layout) {
    if (!t) return fail(CQT_ERR_ARG, "null tables");
    if (batch < 0) return fail(CQT_ERR_ARG, "negative batch");
    if (int rc = check_slices(t, batch)) return rc;
    if (layout != CQT_LAYOUT_PLANAR && layout != CQT_LAYOUT_COMPLEX)
        return fail(CQT_ERR_ARG, "unknown coefficient layout");
    if (batch > 0 && (!ws || ws_bytes < ws_need(t, batch)))
        return fail(CQT_ERR_ARG, "workspace missing or smaller than cqt_workspace_bytes");
    if (((uintptr_t)ws & 15u) != 0) return fail(CQT_ERR_ARG, "workspace not 16-byte aligned");
    return check_device(t);
}

int coef_ptr(const float* re, const float* im, int layout, CoefPtr* out) {
    if (!re) return fail(CQT_ERR_ARG, "null coefficient pointer");
    if (layout == CQT_LAYOUT_PLANAR && !im)
        return fail(CQT_ERR_ARG, "planar layout needs both coefficient planes");
    if (layout == CQT_LAYOUT_COMPLEX && ((uintptr_t)re & 7u))
        return fail(CQT_ERR_ARG, "complex coefficient array not 8-byte aligned");
    out->re = const_cast<float*>(re);
    out->im = const_cast<float*>(im);
    out->interleaved = layout == CQT_LAYOUT_COMPLEX;
    return CQT_OK;
}

BandParams band_params(const cqt_tables* t, int batch) {
    BandParams bp{};
    bp.sc = make_sched(t->ncls, t->cls_M, t->cls_nb, t->cls_first, t->cls_kind, batch);
    bp.tw2048 = t->tw2048;
    bp.twrows = t->twrows;
    bp.ncoef = t->ncoef;
    bp.desc = t->desc;
    bp.ext = t->nbands > kInlineBands;
    std::memcpy(bp.desc_inline, t->desc_host,
                sizeof(int4) * (t->nbands < kInlineBands ? t->nbands : kInlineBands));
    bp.sl = SliceLayout{};
    bp.status = nullptr;
    bp.expire_waits = g_expire_waits.load(std::memory_order_relaxed);
    bp.stride = t->stride;
    return bp;
}

BandParams band_params_sliced(const cqt_tables* t, int rows, int slice0, int slices) {
    BandParams bp = band_params(t, rows * slices);
    bp.sl.S = slices;
    bp.sl.slice0 = slice0;
    long long off = 0;
    for (int g = 0; g < t->ngroups; ++g) {
        bp.sl.goff[g] = off;
        bp.sl.grows[g] = t->group_count[g];
        bp.sl.groll[g] = t->group_roll[g];
        off += (long long)rows * slices * t->group_count[g] * t->group_len[g];
    }
    return bp;
}

SigMap contiguous_in(const float* x) { return SigMap{x, nullptr, 0, 0, 0, 0, 0, 0, nullptr}; }
SigMap contiguous_out(float* y) { return SigMap{nullptr, y, 0, 0, 0, 0, 0, 0, nullptr}; }

// contiguous signals are moved as float2 / float4: null or misaligned rows fail
int check_signal(const float* p, bool input) {
    if (!p) return fail(CQT_ERR_ARG, input ? "null input" : "null output");
    if ((uintptr_t)p & 7u) return fail(CQT_ERR_ARG, "signal not 8-byte aligned");
    return CQT_OK;
}

// one analysis-engine pass: real signal -> spectrum -> bands
int run_fwd(const cqt_tables* t, int which, const SigMap& sig, CoefPtr out,
            BandParams bp, int batch, Scratch sc, cudaStream_t s) {
    if (batch == 0) return CQT_OK;
    float2* X = sc.rows;
    bp.status = sc.status;
    cudaError_t e = launch_spectrum_fwd(sig, X, t->spec, batch, s);
    if (e != cudaSuccess) return cuda_fail(e, "spectrum_fwd launch");
    e = launch_bands_fwd(X, t->fwd[which], bp, out, s);
    if (e != cudaSuccess) return cuda_fail(e, "bands_fwd launch");
    return CQT_OK;
}

int run_fwd_engine(const cqt_tables* t, int which, const float* sig, CoefPtr out,
                   int batch, Scratch sc, cudaStream_t s) {
    return run_fwd(t, which, contiguous_in(sig), out, band_params(t, batch), batch, sc, s);
}

// one synthesis-engine pass: bands -> colour planes -> real signal
int run_inv(const cqt_tables* t, int which, CoefPtr in, const SigMap& sig,
            BandParams bp, int batch, Scratch sc, cudaStream_t s) {
    if (batch == 0) return CQT_OK;
    float2* E = sc.rows;
    bp.status = sc.status;
    cudaError_t e = launch_bands_inv(in, t->inv[which], which, bp, E, s);
    if (e != cudaSuccess) return cuda_fail(e, "bands_inv launch");
    e = launch_spectrum_inv(E, t->inv[which], sig, t->spec, batch, s);
    if (e != cudaSuccess) return cuda_fail(e, "spectrum_inv launch");
    return CQT_OK;
}

int run_inv_engine(const cqt_tables* t, int which, CoefPtr in, float* sig, int batch,
                   void* ws, cudaStream_t s) {
    return run_inv(t, which, in, contiguous_out(sig), band_params(t, batch), batch,
                   scratch_of(ws), s);
}

int sliced_count(long long length) {
    if (length <= 0) return 1;
    const long long nb = (length + kQuarter - 1) / kQuarter;
    return (int)((nb + 1) / 2 + 1);
}

int check_sliced(const cqt_tables* t, const cqt_slices* sl, const cqt_signal* sig, void* ws,
                 size_t ws_bytes) {
    if (!t || !sl || !sig) return fail(CQT_ERR_ARG, "null tables, slicing or signal");
    if (sl->rows < 0 || sl->slices < 1 || sl->slice0 < 0)
        return fail(CQT_ERR_ARG, "bad slicing (rows >= 0, slices >= 1, slice0 >= 0)");
    if (sig->length < 0 || sig->count < 0 || sig->ld < sig->count)
        return fail(CQT_ERR_ARG, "bad signal geometry (length, count >= 0, ld >= count)");
    if (int rc = check_slices(t, (long long)sl->rows * sl->slices)) return rc;
    if (t->ngroups < 1) return fail(CQT_ERR_ARG, "tables carry no group layout");
    if (sl->rows > 0 && (!ws || ws_bytes < ws_need(t, sl->rows * sl->slices)))
        return fail(CQT_ERR_ARG, "workspace missing or smaller than cqt_workspace_bytes(rows * S)");
    if (((uintptr_t)ws & 15u) != 0) return fail(CQT_ERR_ARG, "workspace not 16-byte aligned");
    return check_device(t);
}

SigMap sig_map(const cqt_slices* sl, const cqt_signal* sig, bool input, const float* window) {
    SigMap m{};
    m.x = input ? sig->data : nullptr;
    m.y = input ? nullptr : sig->data;
    m.ld = sig->ld;
    m.length = sig->length;
    m.sample0 = sig->sample0;
    m.count = sig->count;
    m.S = sl->slices;
    m.slice0 = sl->slice0;
    m.window = window;
    return m;
}

}  // namespace

extern "C" {

int cqt_version(void) { return 101; }

const char* cqt_last_error(void) { return g_err.c_str(); }

int cqt_wait_timeouts(unsigned int* count) {
    if (!count) return fail(CQT_ERR_ARG, "null count");
    *count = 0;
    const cudaError_t e = read_wait_timeouts(count);
    return e == cudaSuccess ? CQT_OK : cuda_fail(e, "reading the wait-timeout counter");
}

int cqt_workspace_waits(void* workspace, size_t workspace_bytes, unsigned int* expired,
                        int clear) {
    if (!workspace || !expired || workspace_bytes < kWsHeader)
        return fail(CQT_ERR_ARG, "null workspace or count, or workspace without its header");
    cudaError_t e = cudaMemcpy(expired, workspace, sizeof(unsigned), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "reading the workspace wait status");
    if (clear) {
        e = cudaMemset(workspace, 0, sizeof(unsigned));
        if (e != cudaSuccess) return cuda_fail(e, "clearing the workspace wait status");
    }
    return CQT_OK;
}

int cqt_debug_expire_waits(int on) {
    g_expire_waits.store(on ? 1 : 0, std::memory_order_relaxed);
    return CQT_OK;
}

int32_t cqt_ncoef(const cqt_tables* t) { return t ? t->ncoef : -1; }

int32_t cqt_slice_len(const cqt_tables* t) { return t ? t->nslice : -1; }

// ---- overlap-add halo over peer memory (halo.cu)
struct cqt_halo {
    HaloState st;
};

int cqt_halo_create(int device, int rows, int64_t hop, int wait_ms, cqt_halo** out,
                    void* handle) {
    // one CTA row per signal row: rows <= 65535 (the grid's y extent)
    if (!out || !handle || rows < 1 || rows > 65535 || hop < 1 || wait_ms < 0)
        return fail(CQT_ERR_ARG,
                    "bad halo arguments (1 <= rows <= 65535, hop >= 1, wait_ms >= 0, out, handle)");
    *out = nullptr;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    cqt_halo* h = new cqt_halo{};
    h->st.device = device;
    h->st.rows = rows;
    h->st.hop = hop;
    h->st.wait_ns = (unsigned long long)(wait_ms > 0 ? wait_ms : 10000) * 1000000ull;
    e = halo_create(&h->st, handle);
    if (prev >= 0) cudaSetDevice(prev);
    if (e != cudaSuccess) {
        halo_destroy(&h->st);
        delete h;
        return cuda_fail(e, "halo buffer (cudaMalloc / cudaIpcGetMemHandle)");
    }
    *out = h;
    return CQT_OK;
}

int cqt_halo_connect(cqt_halo* h, const void* left_handle, const void* right_handle) {
    if (!h) return fail(CQT_ERR_ARG, "null halo");
    int prev = -1;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(h->st.device);
    if (e == cudaSuccess && left_handle && !h->st.left) e = halo_open(left_handle, &h->st.left);
    if (e == cudaSuccess && right_handle && !h->st.right)
        e = halo_open(right_handle, &h->st.right);
    if (prev >= 0) cudaSetDevice(prev);
    return e == cudaSuccess ? CQT_OK : cuda_fail(e, "cudaIpcOpenMemHandle(neighbour halo)");
}

int cqt_halo_send(cqt_halo* h, const float* src, int64_t ld, int64_t epoch, void* stream) {
    if (!h || !h->st.left || !src || ld < h->st.hop || epoch < 1)
        return fail(CQT_ERR_ARG, "halo send: not connected to a left neighbour, or bad args");
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev != h->st.device) return fail(CQT_ERR_DEVICE, "halo send: wrong current device");
    const cudaError_t e = halo_send(&h->st, src, ld, epoch, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? CQT_OK : cuda_fail(e, "halo send launch");
}

int cqt_halo_recv_add(cqt_halo* h, float* dst, int64_t ld, int64_t epoch, void* stream) {
    if (!h || !h->st.right || !dst || ld < h->st.hop || epoch < 1)
        return fail(CQT_ERR_ARG, "halo receive: not connected to a right neighbour, or bad args");
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev != h->st.device) return fail(CQT_ERR_DEVICE, "halo receive: wrong current device");
    const cudaError_t e = halo_recv_add(&h->st, dst, ld, epoch, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? CQT_OK : cuda_fail(e, "halo receive launch");
}

int cqt_halo_waits(cqt_halo* h, unsigned int* expired, int clear) {
    if (!h || !expired) return fail(CQT_ERR_ARG, "null halo or count");
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(h->st.device);
    const cudaError_t e = halo_status(&h->st, expired, clear);
    if (prev >= 0) cudaSetDevice(prev);
    return e == cudaSuccess ? CQT_OK : cuda_fail(e, "reading the halo wait status");
}

int cqt_halo_free(cqt_halo* h) {
    if (!h) return CQT_OK;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(h->st.device);
    halo_destroy(&h->st);
    if (prev >= 0) cudaSetDevice(prev);
    delete h;
    return CQT_OK;
}

size_t cqt_workspace_bytes(const cqt_tables* t, int batch) {
    if (!t || batch < 0) return 0;
    return ws_need(t, batch);
}

int cqt_tables_upload(const cqt_host_tables* h, int device, cqt_tables** out) {
    if (!h || !out) return fail(CQT_ERR_ARG, "null argument");
    *out = nullptr;
    // slice geometry (0: the 65536 of the first version of this structure)
    const int nslice = h->slice_len ? h->slice_len : kSlice;
    if (nslice != 65536 && nslice != 32768)
        return fail(CQT_ERR_ARG, "slice length must be 65536 or 32768 samples");
    const int kHalf = nslice / 2, kQuarter = nslice / 4, kPlaneStride = kHalf + 8;
    if (h->nclasses < 1 || h->nclasses > kMaxHostClasses)
        return fail(CQT_ERR_ARG, "class count out of range");
    if (h->sy_nplanes < 1 || h->sy_nplanes > kMaxPlanes || h->aa_nplanes < 1 ||
        h->aa_nplanes > kMaxPlanes)
        return fail(CQT_ERR_ARG, "plane count out of range");
    if (h->ncoef <= 0 || h->nbands <= 0) return fail(CQT_ERR_ARG, "empty tables");
    for (int c = 0; c < h->nclasses; ++c) {
        const int M = h->class_len[c];
        if (M < 16 || M > 2048 || (M & (M - 1)))
            return fail(CQT_ERR_ARG, "block length must be a power of two in 16..2048");
    }
    // host-side bounds check of every table index, so no kernel can read or
    // write outside its buffers whatever tables it is handed
    const int nc = h->ncoef;
    for (int b = 0; b < h->nbands; ++b) {
        if (h->band_list[b] < 0 || h->band_list[b] >= h->nbands)
            return fail(CQT_ERR_ARG, "band_list entry out of range");
        if (h->band_off[b] < 0 || h->band_off[b] > nc)
            return fail(CQT_ERR_ARG, "band offset out of range");
    }
    for (int c = 0; c < h->nclasses; ++c) {
        const int M = h->class_len[c];
        if (h->class_first[c] < 0 || h->class_first[c] + h->class_count[c] > h->nbands)
            return fail(CQT_ERR_ARG, "class range out of band_list");
        for (int i = 0; i < h->class_count[c]; ++i)
            if (h->band_off[h->band_list[h->class_first[c] + i]] + M > nc)
                return fail(CQT_ERR_ARG, "band runs past the heap");
    }
    for (int b = 0; b < h->nbands; ++b) {
        for (const int32_t* sg : {h->an_seg, h->as_seg}) {
            const int lo = sg[2 * b], n = sg[2 * b + 1];
            if (lo < 0 || n < 0 || lo + n > kHalf + 1)
                return fail(CQT_ERR_ARG, "band segment out of the half spectrum");
        }
    }
    for (int c = 0; c < h->nclasses; ++c) {
        const int M = h->class_len[c];
        for (int i = 0; i < h->class_count[c]; ++i) {
            const int b = h->band_list[h->class_first[c] + i];
            const int o = h->band_off[b];
            for (int w = 0; w < 2; ++w) {
                const int32_t* sg = w ? h->as_seg : h->an_seg;
                const int32_t* src = w ? h->as_src : h->an_src;
                const int lo = sg[2 * b], n = sg[2 * b + 1];
                if (n > M) return fail(CQT_ERR_ARG, "band segment longer than its block");
                for (int m = 0; m < M; ++m) {
                    const int s = src[o + m];
                    if (s >= 0 && ((s & 0xFFFF) < lo || (s & 0xFFFF) >= lo + n))
                        return fail(CQT_ERR_ARG, "gather bin outside its band segment");
                }
            }
        }
    }
    if (h->nbands > kMaxBands) return fail(CQT_ERR_ARG, "too many bands");
    // block length of every band, and the group of every band (heap order)
    std::vector<int> band_M(h->nbands, 0), band_group(h->nbands, -1), band_row(h->nbands, 0);
    std::vector<int> group_first(kMaxGroups, 0);
    for (int c = 0; c < h->nclasses; ++c)
        for (int i = 0; i < h->class_count[c]; ++i)
            band_M[h->band_list[h->class_first[c] + i]] = h->class_len[c];
    if (h->ngroups < 1 || h->ngroups > kMaxGroups || !h->group_count || !h->group_roll)
        return fail(CQT_ERR_ARG, "group table missing or too large");
    {
        int b = 0;
        for (int g = 0; g < h->ngroups; ++g) {
            const int n = h->group_count[g];
            if (n < 1 || n > 255 || b + n > h->nbands)
                return fail(CQT_ERR_ARG, "group counts do not partition the bands");
            group_first[g] = b;
            for (int i = 0; i < n; ++i, ++b) {
                band_group[b] = g;
                band_row[b] = i;
                if (band_M[b] != band_M[group_first[g]] ||
                    h->band_off[b] != h->band_off[group_first[g]] + i * band_M[b])
                    return fail(CQT_ERR_ARG, "group bands are not consecutive equal-length rows");
            }
        }
        if (b != h->nbands) return fail(CQT_ERR_ARG, "group counts do not partition the bands");
    }
    // the closed-form octave path must compute exactly what the tables say
    for (int c = 0; c < h->nclasses; ++c) {
        const int M = h->class_len[c];
        for (int i = 0; i < h->class_count[c]; ++i) {
            const int b = h->band_list[h->class_first[c] + i];
            const int32_t* g = h->band_geom + 4 * b;
            if (g[3] & 1) continue;
            const int lo = g[0], l = g[1], lg = g[2];
            const int psy = (g[3] >> 4) & 15, paa = (g[3] >> 8) & 15;
            if (lo < 0 || l < 0 || l >= M || lg < 0 || lg > M || lo + lg > kHalf + 1 ||
                psy >= h->sy_nplanes || paa >= h->aa_nplanes)
                return fail(CQT_ERR_ARG, "band geometry out of range");
            const int o = h->band_off[b];
            for (int m = 0; m < M; ++m) {
                const int ii = (m + l) & (M - 1);
                const bool in_win = ii < lg;
                const int bin = lo + ii;
                for (int w = 0; w < 2; ++w) {   // analysis-engine sets
                    const int s = (w ? h->as_src : h->an_src)[o + m];
                    const float gn = (w ? h->as_gain : h->an_gain)[o + m];
                    const bool ok = s >= 0 ? (in_win && s == bin) : gn == 0.f;
                    if (!ok) return fail(CQT_ERR_ARG, "octave gather table disagrees with geometry");
                }
                for (int w = 0; w < 2; ++w) {   // synthesis-engine sets
                    const int32_t* dst = w ? h->aa_dest : h->sy_dest;
                    const float gr = (w ? h->aa_gre : h->sy_gre)[o + m];
                    const float gi = (w ? h->aa_gim : h->sy_gim)[o + m];
                    const uint8_t* mk = w ? h->aa_mask : h->sy_mask;
                    const int pl = w ? paa : psy;
                    const bool writes = in_win && gr != 0.f;
                    if (writes != (dst[o + m] >= 0))
                        return fail(CQT_ERR_ARG, "octave scatter table disagrees with geometry");
                    if (writes && (dst[o + m] != pl * kPlaneStride + bin || gi != gr ||
                                   !((mk[bin] >> pl) & 1)))
                        return fail(CQT_ERR_ARG, "octave scatter slot disagrees with geometry");
                }
            }
        }
    }
    for (int i = 0; i < nc; ++i) {
        for (const int32_t* s : {h->an_src, h->as_src})
            if (s[i] >= 0 && ((s[i] & 0xFFFF) > kHalf || (s[i] & ~0x1FFFF)))
                return fail(CQT_ERR_ARG, "gather bin out of range");
        if (h->sy_dest[i] >= h->sy_nplanes * kPlaneStride ||
            h->aa_dest[i] >= h->aa_nplanes * kPlaneStride ||
            (h->sy_dest[i] >= 0 && h->sy_dest[i] % kPlaneStride > kHalf) ||
            (h->aa_dest[i] >= 0 && h->aa_dest[i] % kPlaneStride > kHalf))
            return fail(CQT_ERR_ARG, "scatter slot out of range");
    }

    for (int q = 0; q < kPlaneStride; ++q)
        if ((h->sy_mask[q] >> h->sy_nplanes) || (h->aa_mask[q] >> h->aa_nplanes) ||
            (q > kHalf && (h->sy_mask[q] | h->aa_mask[q])))
            return fail(CQT_ERR_ARG, "plane mask names a plane or bin out of range");

    // internal classes: each host class's octave bands (pruned when the
    // first-stage inputs r = 6..9 of every radix-16 butterfly lie outside
    // every band's window support), then its side bands; the host classes
    // must cover every band exactly once
    std::vector<int> order;
    std::vector<int> seen(h->nbands, 0);
    int ncls = 0, cls_M[kMaxClasses], cls_nb[kMaxClasses], cls_first[kMaxClasses],
        cls_kind[kMaxClasses];
    for (int c = 0; c < h->nclasses; ++c) {
        const int M = h->class_len[c];
        for (int kind = 0; kind < 2; ++kind) {
            const int first = (int)order.size();
            bool prune = true;
            for (int i = 0; i < h->class_count[c]; ++i) {
                const int b = h->band_list[h->class_first[c] + i];
                const int32_t* g = h->band_geom + 4 * b;
                if ((int)(g[3] & 1) != kind) continue;
                if (seen[b]++) return fail(CQT_ERR_ARG, "a band sits in two classes");
                order.push_back(b);
                for (int r = 6; r <= 9 && kind == 0; ++r)
                    for (int j = 0; j < M / 16; ++j)
                        if (((j + r * (M / 16) + g[1]) & (M - 1)) < g[2]) prune = false;
            }
            const int nb = (int)order.size() - first;
            if (nb == 0) continue;
            cls_M[ncls] = M;
            cls_nb[ncls] = nb;
            cls_first[ncls] = first;
            cls_kind[ncls] = kind ? kSide : (prune ? kOctavePruned : kOctave);
            ++ncls;
        }
    }
    if ((int)order.size() != h->nbands) return fail(CQT_ERR_ARG, "classes do not cover every band");

    int prev = -1;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");

    // one blob: [int32 arrays][float arrays][uint8 masks][float2 twiddles]
    struct Part { const void* src; size_t bytes; size_t off; };
    std::vector<Part> parts;
    size_t total = 0;
    auto add = [&](const void* p, size_t bytes) {
        total = (total + 255) & ~(size_t)255;
        parts.push_back({p, bytes, total});
        total += bytes;
        return parts.size() - 1;
    };
    const size_t nI = (size_t)nc * 4, nB = (size_t)h->nbands * 4;
    const size_t maskB = (size_t)kPlaneStride;
    size_t i_boff = add(h->band_off, nB), i_blist = add(h->band_list, nB);
    size_t i_ans = add(h->an_src, nI), i_ang = add(h->an_gain, nI);
    size_t i_ass = add(h->as_src, nI), i_asg = add(h->as_gain, nI);
    size_t i_ansg = add(h->an_seg, nB * 2), i_assg = add(h->as_seg, nB * 2);
    size_t i_syd = add(h->sy_dest, nI), i_syr = add(h->sy_gre, nI), i_syi = add(h->sy_gim, nI);
    size_t i_sym = add(h->sy_mask, maskB);
    size_t i_aad = add(h->aa_dest, nI), i_aar = add(h->aa_gre, nI), i_aai = add(h->aa_gim, nI);
    size_t i_aam = add(h->aa_mask, maskB);
    // quad masks of the inverse spectrum engine
    std::vector<uint16_t> qm_sy(kQuarter / 2 + 1), qm_aa(kQuarter / 2 + 1);
    for (int n = 0; n <= kQuarter / 2; ++n) {
        const int bins[4] = {n, kHalf - n, kQuarter + n, kQuarter - n};
        uint16_t a = 0, b = 0;
        for (int k = 0; k < 4; ++k) {
            a |= (uint16_t)((h->sy_mask[bins[k]] & 15) << (4 * k));
            b |= (uint16_t)((h->aa_mask[bins[k]] & 15) << (4 * k));
        }
        qm_sy[n] = a;
        qm_aa[n] = b;
    }
    size_t i_qsy = add(qm_sy.data(), qm_sy.size() * 2), i_qaa = add(qm_aa.data(), qm_aa.size() * 2);
    // band descriptors in class order (see BandParams)
    std::vector<int4> desc(h->nbands);
    for (int i = 0; i < h->nbands; ++i) {
        const int b = order[i];
        const int32_t* g = h->band_geom + 4 * b;
        const bool side = g[3] & 1;
        desc[i] = make_int4(h->band_off[b], side ? b : g[0], g[1] | (g[2] << 16),
                            (g[3] & 0xFFF) | (band_group[b] << 12) | (band_row[b] << 16));
    }
    size_t i_desc = add(desc.data(), desc.size() * sizeof(int4));
    size_t i_tw = add(h->tw2048, 2048 * 8), i_hi = add(h->tw_hi, 256 * 8), i_lo = add(h->tw_lo, 256 * 8);
    std::vector<float2> rows(spectrum_twiddle_count());
    spectrum_twiddle_rows(rows.data());
    size_t i_rows = add(rows.data(), rows.size() * sizeof(float2));
    std::vector<float2> twrows(band_twiddle_count());
    band_twiddle_rows(twrows.data(), reinterpret_cast<const float2*>(h->tw2048));
    size_t i_twr = add(twrows.data(), twrows.size() * sizeof(float2));

    void* blob = nullptr;
    e = cudaMalloc(&blob, total);
    if (e != cudaSuccess) {
        cudaSetDevice(prev);
        return cuda_fail(e, "cudaMalloc(tables)");
    }
    for (const Part& p : parts) {
        e = cudaMemcpy(static_cast<char*>(blob) + p.off, p.src, p.bytes, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            cudaFree(blob);
            cudaSetDevice(prev);
            return cuda_fail(e, "cudaMemcpy(tables)");
        }
    }
    e = init_spectrum_attributes();
    if (e == cudaSuccess) e = init_band_attributes();
    if (e != cudaSuccess) {
        cudaFree(blob);
        cudaSetDevice(prev);
        return cuda_fail(e, "cudaFuncSetAttribute");
    }

    auto P = [&](size_t i) { return static_cast<char*>(blob) + parts[i].off; };
    cqt_tables* t = new cqt_tables{};
    t->device = device;
    t->ncoef = nc;
    t->nbands = h->nbands;
    t->ncls = ncls;
    for (int c = 0; c < ncls; ++c) {
        t->cls_M[c] = cls_M[c];
        t->cls_nb[c] = cls_nb[c];
        t->cls_first[c] = cls_first[c];
        t->cls_kind[c] = cls_kind[c];
    }
    t->fwd[0] = FwdTab{(const int*)P(i_ans), (const float*)P(i_ang), (const int2*)P(i_ansg)};
    t->fwd[1] = FwdTab{(const int*)P(i_ass), (const float*)P(i_asg), (const int2*)P(i_assg)};
    t->inv[0] = InvTab{(const int*)P(i_syd), (const float*)P(i_syr), (const float*)P(i_syi),
                       (const unsigned char*)P(i_sym), (const unsigned short*)P(i_qsy),
                       h->sy_nplanes};
    t->inv[1] = InvTab{(const int*)P(i_aad), (const float*)P(i_aar), (const float*)P(i_aai),
                       (const unsigned char*)P(i_aam), (const unsigned short*)P(i_qaa),
                       h->aa_nplanes};
    t->tw2048 = (const float2*)P(i_tw);
    t->twrows = (const float2*)P(i_twr);
    t->ngroups = h->ngroups;
    for (int g = 0; g < h->ngroups; ++g) {
        t->group_count[g] = h->group_count[g];
        t->group_roll[g] = h->group_roll[g] ? 1 : 0;
        t->group_len[g] = band_M[group_first[g]];
    }
    t->desc = (const int4*)P(i_desc);
    for (int i = 0; i < h->nbands && i < kInlineBands; ++i) t->desc_host[i] = desc[i];
    t->spec = SpecTables{(const float2*)P(i_hi), (const float2*)P(i_lo), (const float2*)P(i_rows),
                         nslice};
    t->max_planes = h->sy_nplanes > h->aa_nplanes ? h->sy_nplanes : h->aa_nplanes;
    t->nslice = nslice;
    t->half = kHalf;
    t->quarter = kQuarter;
    t->stride = kPlaneStride;
    t->spec.nslice = nslice;
    t->blob = blob;
    *out = t;
    if (prev >= 0) cudaSetDevice(prev);
    return CQT_OK;
}

int cqt_tables_free(cqt_tables* t) {
    if (!t) return CQT_OK;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(t->device);
    cudaError_t e = cudaFree(t->blob);
    if (prev >= 0) cudaSetDevice(prev);
    delete t;
    return e == cudaSuccess ? CQT_OK : cuda_fail(e, "cudaFree(tables)");
}

int cqt_analysis(const cqt_tables* t, const float* x, float* c_re, float* c_im, int layout,
                 int batch, void* ws, size_t ws_bytes, void* stream) {
    int rc = check_common(t, batch, ws, ws_bytes, layout);
    if (rc) return rc;
    if (batch && (rc = check_signal(x, true))) return rc;
    CoefPtr out;
    if (batch && (rc = coef_ptr(c_re, c_im, layout, &out))) return rc;
    return run_fwd_engine(t, 0, x, out, batch, scratch_of(ws), static_cast<cudaStream_t>(stream));
}

int cqt_adj_synthesis(const cqt_tables* t, const float* gy, float* g_re, float* g_im,
                      int layout, int batch, void* ws, size_t ws_bytes, void* stream) {
    int rc = check_common(t, batch, ws, ws_bytes, layout);
    if (rc) return rc;
    if (batch && (rc = check_signal(gy, true))) return rc;
    CoefPtr out;
    if (batch && (rc = coef_ptr(g_re, g_im, layout, &out))) return rc;
    return run_fwd_engine(t, 1, gy, out, batch, scratch_of(ws), static_cast<cudaStream_t>(stream));
}

int cqt_synthesis(const cqt_tables* t, const float* c_re, const float* c_im, int layout,
                  float* y, int batch, void* ws, size_t ws_bytes, void* stream) {
    int rc = check_common(t, batch, ws, ws_bytes, layout);
    if (rc) return rc;
    if (batch && (rc = check_signal(y, false))) return rc;
    CoefPtr in;
    if (batch && (rc = coef_ptr(c_re, c_im, layout, &in))) return rc;
    return run_inv_engine(t, 0, in, y, batch, ws, static_cast<cudaStream_t>(stream));
}

int cqt_adj_analysis(const cqt_tables* t, const float* g_re, const float* g_im, int layout,
                     float* gx, int batch, void* ws, size_t ws_bytes, void* stream) {
    int rc = check_common(t, batch, ws, ws_bytes, layout);
    if (rc) return rc;
    if (batch && (rc = check_signal(gx, false))) return rc;
    CoefPtr in;
    if (batch && (rc = coef_ptr(g_re, g_im, layout, &in))) return rc;
    return run_inv_engine(t, 1, in, gx, batch, ws, static_cast<cudaStream_t>(stream));
}

int cqt_synthesis_sqerr(const cqt_tables* t, const float* c_re, const float* c_im, int layout,
                        float* y, const float* target, float* loss, float loss_scale,
                        int batch, void* ws, size_t ws_bytes, void* stream) {
    int rc = check_common(t, batch, ws, ws_bytes, layout);
    if (rc) return rc;
    if (!loss) return fail(CQT_ERR_ARG, "null loss");
    if (((uintptr_t)loss & 3u) != 0) return fail(CQT_ERR_ARG, "loss not 4-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (batch > 0) {
        if ((rc = check_signal(y, false))) return rc;
        if ((rc = check_signal(target, true))) return rc;
        CoefPtr in;
        if ((rc = coef_ptr(c_re, c_im, layout, &in))) return rc;
        SigMap out = contiguous_out(y);
        out.target = target;
        out.partial = ws_partials(t, batch, ws);
        if ((rc = run_inv(t, 0, in, out, band_params(t, batch), batch, scratch_of(ws), s)))
            return rc;
    }
    // an empty batch still defines the loss: the sum of nothing
    cudaError_t e = launch_sqerr_finish(batch > 0 ? ws_partials(t, batch, ws) : nullptr,
                                        spectrum_ctas(batch), loss_scale, loss, s);
    return e == cudaSuccess ? CQT_OK : cuda_fail(e, "squared-error sum launch");
}

int cqt_adj_synthesis_sqerr(const cqt_tables* t, const float* y, const float* target,
                            float scale, const float* scale_dev, float* g_re, float* g_im,
                            int layout, int batch, void* ws, size_t ws_bytes, void* stream) {
    int rc = check_common(t, batch, ws, ws_bytes, layout);
    if (rc) return rc;
    if (batch == 0) return CQT_OK;
    if ((rc = check_signal(y, true))) return rc;
    if ((rc = check_signal(target, true))) return rc;
    if (((uintptr_t)scale_dev & 3u) != 0) return fail(CQT_ERR_ARG, "scale_dev not 4-byte aligned");
    CoefPtr out;
    if ((rc = coef_ptr(g_re, g_im, layout, &out))) return rc;
    SigMap in = contiguous_in(y);
    in.target = target;
    in.scale_dev = scale_dev;
    in.scale = scale;
    return run_fwd(t, 1, in, out, band_params(t, batch), batch, scratch_of(ws),
                   static_cast<cudaStream_t>(stream));
}

int cqt_launch_stage(const cqt_tables* t, int stage, const float* sig_in, float* sig_out,
                     float* c_re, float* c_im, int layout, int batch, void* ws,
                     size_t ws_bytes, void* stream) {
    int rc = check_common(t, batch, ws, ws_bytes, layout);
    if (rc) return rc;
    if (batch == 0) return CQT_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    CoefPtr cp;
    const Scratch sc = scratch_of(ws);
    BandParams bp = band_params(t, batch);
    bp.status = sc.status;
    switch (stage) {
    case 0:
        if ((rc = check_signal(sig_in, true))) return rc;
        e = launch_spectrum_fwd(contiguous_in(sig_in), sc.rows, t->spec, batch, s);
        break;
    case 1:
        if ((rc = coef_ptr(c_re, c_im, layout, &cp))) return rc;
        e = launch_bands_fwd(sc.rows, t->fwd[0], bp, cp, s);
        break;
    case 2:
        if ((rc = coef_ptr(c_re, c_im, layout, &cp))) return rc;
        e = launch_bands_inv(cp, t->inv[0], 0, bp, sc.rows, s);
        break;
    case 3:
        if ((rc = check_signal(sig_out, false))) return rc;
        e = launch_spectrum_inv(sc.rows, t->inv[0], contiguous_out(sig_out), t->spec, batch, s);
        break;
    default:
        return fail(CQT_ERR_ARG, "unknown stage");
    }
    return e == cudaSuccess ? CQT_OK : cuda_fail(e, "stage launch");
}

}  // extern "C"

// ------------------------------------------------------------------------
// Allocation-free analysis.
//
// Some callers cannot allocate device memory at all: a real-time audio
// callback (a plugin's process() on the host's audio thread) must not call
// cudaMalloc, which can block and synchronise the device and so cause audio
// dropouts, and a host with a fixed, pre-planned memory budget may forbid
// allocations after start-up.  cqt_analysis_noalloc serves them: it is
// cqt_analysis with its scratch (the half-spectrum rows of the slices) taken
// from the file-scope array below instead of a caller-allocated workspace.
//
// * The array holds at most kNoAllocMaxBatch = 8 slices (2,097,664 bytes);
//   every GPU that loads this library keeps it until the process exits.
// * The first call on a device, with that device current, looks up the
//   array's device address with cudaGetSymbolAddress and caches it.  That
//   lookup may make the CUDA runtime load this library's device code (lazy
//   module loading), which can itself allocate and synchronise; so make one
//   warm-up call per device at start-up, off the real-time thread and before
//   any stream capture (batch 0 is enough: the lookup comes before the
//   empty-batch return).  Later calls take the cached address with one atomic
//   load, no lock, and allocate nothing.
// * All calls on a device share the array and it keeps the last call's
//   contents.  Nothing in it needs clearing (the spectrum kernel writes every
//   bin the band kernel later reads), but calls that overlap on the GPU --
//   e.g. on two streams without ordering between them -- race on it.
namespace {

constexpr int kNoAllocMaxBatch = 8;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) float2 g_noalloc_scratch[kNoAllocMaxBatch * kPlaneStride];

std::mutex g_noalloc_mu;                              // first lookup per device only
std::atomic<void*> g_noalloc_ptr[kNoAllocMaxDevices];

}  // namespace

extern "C" int cqt_analysis_noalloc(const cqt_tables* t, const float* x, float* c_re,
                                    float* c_im, int layout, int batch, void* stream) {
    if (!t) return fail(CQT_ERR_ARG, "null tables");
    if (batch < 0) return fail(CQT_ERR_ARG, "negative batch");
    if (batch > kNoAllocMaxBatch)
        return fail(CQT_ERR_ARG,
                    "cqt_analysis_noalloc takes at most 8 slices per call (its static "
                    "scratch holds 8); split the batch or use cqt_analysis");
    if (layout != CQT_LAYOUT_PLANAR && layout != CQT_LAYOUT_COMPLEX)
        return fail(CQT_ERR_ARG, "unknown coefficient layout");
    int rc = check_device(t);
    if (rc) return rc;
    if (t->device < 0 || t->device >= kNoAllocMaxDevices)
        return fail(CQT_ERR_DEVICE, "device index beyond the no-allocation address cache");
    void* scratch = g_noalloc_ptr[t->device].load(std::memory_order_acquire);
    if (!scratch) {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        scratch = g_noalloc_ptr[t->device].load(std::memory_order_relaxed);
        if (!scratch) {
            cudaError_t e = cudaGetSymbolAddress(&scratch, g_noalloc_scratch);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
            g_noalloc_ptr[t->device].store(scratch, std::memory_order_release);
        }
    }
    if (batch == 0) return CQT_OK;
    if ((rc = check_signal(x, true))) return rc;
    CoefPtr out;
    if ((rc = coef_ptr(c_re, c_im, layout, &out))) return rc;
    return run_fwd_engine(t, 0, x, out, batch, Scratch{static_cast<float2*>(scratch), nullptr},
                          static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------------------
// Sliced streaming transform (include/flash_cqt_b200.h): the SlicedCQT
// slicing, rolls and overlap-add folded into the same four kernels.
extern "C" {

int cqt_sliced_count(int64_t length) { return sliced_count(length); }

int cqt_sliced_analysis(const cqt_tables* t, const cqt_signal* x, const cqt_slices* sl,
                        float* coef, void* ws, size_t ws_bytes, void* stream) {
    int rc = check_sliced(t, sl, x, ws, ws_bytes);
    if (rc) return rc;
    if (sl->rows == 0) return CQT_OK;
    if (!x->data || !coef || !sl->window)
        return fail(CQT_ERR_ARG, "null signal, coefficients or window");
    if ((uintptr_t)coef & 7u) return fail(CQT_ERR_ARG, "coefficient buffer not 8-byte aligned");
    const CoefPtr out{coef, nullptr, 1};
    return run_fwd(t, 0, sig_map(sl, x, true, sl->window), out,
                   band_params_sliced(t, sl->rows, sl->slice0, sl->slices),
                   sl->rows * sl->slices, scratch_of(ws), static_cast<cudaStream_t>(stream));
}

int cqt_sliced_adj_synthesis(const cqt_tables* t, const cqt_signal* gy, const cqt_slices* sl,
                             float* gcoef, void* ws, size_t ws_bytes, void* stream) {
    int rc = check_sliced(t, sl, gy, ws, ws_bytes);
    if (rc) return rc;
    if (sl->rows == 0) return CQT_OK;
    if (!gy->data || !gcoef) return fail(CQT_ERR_ARG, "null gradient buffers");
    if ((uintptr_t)gcoef & 7u) return fail(CQT_ERR_ARG, "coefficient buffer not 8-byte aligned");
    const CoefPtr out{gcoef, nullptr, 1};
    return run_fwd(t, 1, sig_map(sl, gy, true, nullptr), out,
                   band_params_sliced(t, sl->rows, sl->slice0, sl->slices),
                   sl->rows * sl->slices, scratch_of(ws), static_cast<cudaStream_t>(stream));
}

static int sliced_inv(const cqt_tables* t, int which, const float* coef, const cqt_slices* sl,
                      const float* window, const cqt_signal* y, void* ws, size_t ws_bytes,
                      void* stream) {
    int rc = check_sliced(t, sl, y, ws, ws_bytes);
    if (rc) return rc;
    if (sl->rows == 0) return CQT_OK;
    if (!coef || !y->data) return fail(CQT_ERR_ARG, "null coefficients or output");
    if ((uintptr_t)coef & 7u) return fail(CQT_ERR_ARG, "coefficient buffer not 8-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // overlap-add target: zero the rows first (stream-ordered, capturable)
    if (y->count > 0) {
        cudaError_t e = cudaMemset2DAsync(y->data, (size_t)y->ld * sizeof(float), 0,
                                          (size_t)y->count * sizeof(float), sl->rows, s);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemset2DAsync(overlap-add target)");
    }
    const CoefPtr in{const_cast<float*>(coef), nullptr, 1};
    return run_inv(t, which, in, sig_map(sl, y, false, window),
                   band_params_sliced(t, sl->rows, sl->slice0, sl->slices),
                   sl->rows * sl->slices, scratch_of(ws), s);
}

int cqt_sliced_synthesis(const cqt_tables* t, const float* coef, const cqt_slices* sl,
                         const cqt_signal* y, void* ws, size_t ws_bytes, void* stream) {
    return sliced_inv(t, 0, coef, sl, nullptr, y, ws, ws_bytes, stream);
}

int cqt_sliced_adj_analysis(const cqt_tables* t, const float* gcoef, const cqt_slices* sl,
                            const cqt_signal* gx, void* ws, size_t ws_bytes, void* stream) {
    if (!sl || !sl->window)
        return fail(CQT_ERR_ARG, "the transpose of the sliced analysis needs the window");
    return sliced_inv(t, 1, gcoef, sl, sl->window, gx, ws, ws_bytes, stream);
}

}  // extern "C"
