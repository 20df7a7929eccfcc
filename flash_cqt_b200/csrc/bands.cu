// Band engine: the per-band native-length transforms of the constant-Q
// analysis and synthesis (block lengths M = 32 ... 2048, 154 bands a slice).
//
// bands_fwd (analysis engine; also the transpose of the synthesis):
//   gather   v[m] = gain[m] * X~[bin(m)]          (window / routing)
//   DFT      coef[n] = sum_m v[m] e^{+2 pi i m n / M}   (1/M folded in gain)
//   store    natural-order coefficient heap, coalesced
// bands_inv (synthesis engine; also the transpose of the analysis):
//   load     coefficient heap, coalesced
//   DFT      S[m] = sum_n coef[n] e^{-2 pi i m n / M}
//   scatter  E[plane, bin(m)] = (Re S gre[m], Im S gim[m])  one owned slot per tap
//
// Octave bands (all but the DC and Nyquist side bands) have a closed-form
// tap -> bin map: tap m reads / writes bin lo + ((m + l) mod M), live when
// (m + l) mod M < Lg (the window support, oct_cqt.py:44-58), no conjugation,
// one colour plane per band -- so they need one gain load per tap and no
// index tables.  The two side bands take the table path (src / dest tables,
// conjugated mirror taps).  Band descriptors come from the kernel
// parameters (the first 160) or the table blob.
//
// Replaces the reference's radix band engine (radix_impl.cuh:146-443: warp
// shuffle radix-8/16/32 butterflies, one CTA per (band, slice), atomics in
// the inverse): here each thread holds 32 points in registers and runs whole
// radix-2..32 butterflies, stages exchange through padded shared memory, the
// inter-stage twiddles sit in conflict-free shared rows, and one 256-thread
// CTA processes 8192 points = 8192 / M (band, slice) instances of one block
// length so small bands batch up.
#include <cstdint>

#include "engine.cuh"
#include "internal.h"

namespace fcqt {

namespace {

#ifndef FCQT_PREFETCH_GAINS
#define FCQT_PREFETCH_GAINS 0
#endif

constexpr int kP = kBandP;
constexpr int kSH = kP == 32 ? 5 : 4;                    // shared padding shift
// shared-memory stride of one (band, slice) instance: the padded length
// rounded up to an even number of float2, so that every instance buffer
// starts on a 16-byte boundary (TMA bulk copies need it; with kSH = 5 and
// M = 32 the padded length, 33, is odd)
constexpr int inst_stride(int M) { return (padded<kSH>(M) + 1) & ~1; }
constexpr int data_need(int M) { return M > kBandCap ? 0 : (kBandCap / M) * inst_stride(M); }
constexpr int cmax(int a, int b) { return a > b ? a : b; }
constexpr int kBandData =                                 // float2 per CTA
    cmax(cmax(cmax(cmax(data_need(16), data_need(32)), data_need(64)),
              cmax(data_need(128), data_need(256))),
         cmax(cmax(data_need(512), data_need(1024)), data_need(2048)));
static_assert(kBandData >= padded<kSH>(kBandCap), "instance buffers overlap");
// Build-time tuning switches (defaults are the measured best):
//   FCQT_TW3_SMEM   stage-3 twiddles as shared rows (1) or from the global
//                   W_2048 table (0: less shared memory per CTA, faster);
//   FCQT_TW3_POW    stage-3 twiddles W^k, W^2k, W^4k and their products (1);
//   FCQT_PREFETCH_GAINS  bands_inv loads its scatter gains before the stages
//                   (1), or in the scatter (0: with the twiddles in shared
//                   slots, 5 % faster -- the early loads cost registers).
#ifndef FCQT_TW3_SMEM
#define FCQT_TW3_SMEM 0
#endif
constexpr int kBandTw = FCQT_TW3_SMEM ? 2048 : 1024;     // >= largest twiddle set
constexpr int kBandSmem = (kBandData + kBandTw) * 8;
// resident CTAs per SM at 128 (P = 32) or 64 (P = 16) registers a thread
constexpr int kBandMinBlocks = (kP == 32 ? 2 : 4) * 256 / kBandThreads;

template <int M, int P = kP> struct Sched;   // stage radices per block length
// (only the build's own points-per-thread set is compiled in)
#if FCQT_BAND_P == 32
template <> struct Sched<32, 32>   { static constexpr int R1 = 32, R2 = 1,  R3 = 1; };
template <> struct Sched<64, 32>   { static constexpr int R1 = 32, R2 = 2,  R3 = 1; };
template <> struct Sched<128, 32>  { static constexpr int R1 = 32, R2 = 4,  R3 = 1; };
template <> struct Sched<256, 32>  { static constexpr int R1 = 32, R2 = 8,  R3 = 1; };
template <> struct Sched<512, 32>  { static constexpr int R1 = 32, R2 = 16, R3 = 1; };
template <> struct Sched<1024, 32> { static constexpr int R1 = 32, R2 = 32, R3 = 1; };
template <> struct Sched<2048, 32> { static constexpr int R1 = 32, R2 = 32, R3 = 2; };
#else
template <> struct Sched<16, 16>   { static constexpr int R1 = 16, R2 = 1,  R3 = 1; };
template <> struct Sched<32, 16>   { static constexpr int R1 = 16, R2 = 2,  R3 = 1; };
template <> struct Sched<64, 16>   { static constexpr int R1 = 16, R2 = 4,  R3 = 1; };
template <> struct Sched<128, 16>  { static constexpr int R1 = 16, R2 = 8,  R3 = 1; };
template <> struct Sched<256, 16>  { static constexpr int R1 = 16, R2 = 16, R3 = 1; };
template <> struct Sched<512, 16>  { static constexpr int R1 = 16, R2 = 16, R3 = 2; };
template <> struct Sched<1024, 16> { static constexpr int R1 = 16, R2 = 16, R3 = 4; };
template <> struct Sched<2048, 16> { static constexpr int R1 = 16, R2 = 16, R3 = 8; };
#endif

// shared twiddle rows of one block length: stage 2 rows W_{NS R}^{r k}
// (r = 1..R2-1, k < NS2 = R1), then stage 3 rows (r = 1..R3-1, k < R1 R2)
template <int M>
struct TwLayout {
    static constexpr int R1 = Sched<M>::R1, R2 = Sched<M>::R2, R3 = Sched<M>::R3;
    static constexpr int n2 = (R2 - 1) * R1;
    static constexpr int n3 = FCQT_TW3_SMEM ? (R3 - 1) * R1 * R2 : 0;
    static_assert(n2 + n3 <= kBandTw, "twiddle rows exceed their shared slot");
};

// Build-time switch FCQT_TW_TMA (1): every twiddle a band CTA reads in its
// stages -- the stage-2 rows and the last stage's base powers W^k, W^2k, W^4k
// -- sits in a per-length slot of a table in the device blob, laid out as
// the CTA's shared slot, and arrives with one TMA bulk copy on the staging
// barrier (0: the CTA's threads gather the stage-2 rows from W_2048 and the
// last stage reads its powers from global memory per butterfly).  Both give
// the same values: the slots are copied from the same W_2048 table.
#ifndef FCQT_TW_TMA
// the 32-point-per-thread build's M = 2048 schedule (32 x 32 x 2) needs 2016
// twiddle entries, more than the slot holds: it gathers them as before
#define FCQT_TW_TMA (FCQT_BAND_P <= 16)
#endif
static_assert(!(FCQT_TW_TMA && FCQT_TW3_SMEM), "one place for the last-stage twiddles");

template <int M>
struct TwSlot {
    using L = TwLayout<M>;
    static constexpr int NS3 = L::R1 * L::R2;   // span of the last stage
    static constexpr int npow = L::R3 >= 8 ? 3 : L::R3 >= 4 ? 2 : L::R3 >= 2 ? 1 : 0;
    static constexpr int count = L::n2 + npow * NS3;   // float2
    static constexpr unsigned bytes = count * 8u;
    static_assert(!FCQT_TW_TMA || (count <= kBandTw && bytes % 16u == 0),
                  "twiddle slot too small or unaligned");
};
// slot of block length M (16, 32, ..., 2048) in the table
constexpr int tw_slot_index(int M) {
    return M <= 16 ? 0 : M == 32 ? 1 : M == 64 ? 2 : M == 128 ? 3 : M == 256 ? 4
           : M == 512 ? 5 : M == 1024 ? 6 : 7;
}
constexpr int kTwSlots = 8;

template <int M>
__device__ __forceinline__ void fill_twiddles(float2* tws, const float2* __restrict__ w2048) {
    using L = TwLayout<M>;
    constexpr int NT = (L::n2 + L::n3 + kBandThreads - 1) / kBandThreads;
#pragma unroll
    for (int it = 0; it < NT; ++it) {
        const int e = threadIdx.x + it * kBandThreads;
        if (e >= L::n2 + L::n3) break;
        int r, k, span, R;
        if (e < L::n2) {
            r = e / L::R1 + 1;
            k = e % L::R1;
            span = L::R1;
            R = L::R2;
        } else {
            const int f = e - L::n2;
            span = L::R1 * L::R2;
            R = L::R3;
            r = f / span + 1;
            k = f % span;
        }
        tws[e] = __ldg(w2048 + ((r * k * (2048 / (span * R))) & 2047));
    }
}

// Twiddle (span NS > 1) and DFT for all butterflies of a thread; twiddles
// from shared rows (row r - 1 at rows + (r - 1) NS), conjugated for S = +1
template <int M, int T, int R, int NS, int S, int P>
__device__ __forceinline__ void stage_compute_rows(float2 (&v)[P], int t, const float2* rows) {
    static_for<0, P / R>([&](auto Bb) {
        constexpr int b = decltype(Bb)::value;
        if constexpr (NS > 1) {
            const int k = (t + T * b) % NS;
#pragma unroll
            for (int r = 1; r < R; ++r) {
                float2 w = rows[(r - 1) * NS + k];
                if constexpr (S > 0) w.y = -w.y;
                v[b * R + r] = cmul(v[b * R + r], w);
            }
        }
        dft<R, S, b * R, 1>(v);
    });
}

struct Inst {
    int t;        // thread index within the instance
    int il;       // instance index within the CTA
    bool valid;
    int slice;
    int4 d;       // band descriptor
};

template <int M, bool EXT>
__device__ __forceinline__ Inst locate(const BandParams& bp, int c) {
    constexpr int T = M / kP;
    constexpr int IPC = kBandThreads / T;
    Inst in;
    in.t = threadIdx.x % T;
    in.il = threadIdx.x / T;
    const int inst = (blockIdx.x - bp.sc.cta0[c]) * IPC + in.il;
    const int B = bp.sc.batch;
    in.valid = inst < bp.sc.nb[c] * B;
    // inst / B by a float reciprocal (inst < 2^24) and one correction step
    int q = __float2int_rz(__int2float_rn(inst) * bp.sc.inv_batch);
    int rem = inst - q * B;
    if (rem >= B) { ++q; rem -= B; }
    if (rem < 0) { --q; rem += B; }
    in.slice = in.valid ? rem : 0;
    const int di = bp.sc.first[c] + (in.valid ? q : 0);
    // banks within kInlineBands read the parameters, larger ones device memory
    if constexpr (EXT)
        in.d = __ldg(bp.desc + di);
    else
        in.d = bp.desc_inline[di];
    return in;
}

#ifndef FCQT_TW3_POW
#define FCQT_TW3_POW 1
#endif

// Last-stage twiddles W^{r k} (r < R <= 8) from W^k, W^2k and W^4k only:
// the other powers are products of at most two of them (two roundings)
template <int M, int T, int R, int NS, int S, int TWBASE, int P, class TW>
__device__ __forceinline__ void stage_compute_pow(float2 (&v)[P], int t, const TW& tw) {
    static_assert(R == 2 || R == 4 || R == 8, "power twiddles for radix 2, 4, 8");
    static_for<0, P / R>([&](auto Bb) {
        constexpr int b = decltype(Bb)::value;
        const int k = (t + T * b) % NS;
        constexpr int scale = TWBASE / (NS * R);
        static_assert(scale * NS * R == TWBASE, "twiddle base too small");
        float2 w[R];
        w[1] = tw(k * scale);
        if constexpr (R >= 4) {
            w[2] = tw(2 * k * scale);
            w[3] = cmul(w[1], w[2]);
        }
        if constexpr (R == 8) {
            w[4] = tw(4 * k * scale);
            w[5] = cmul(w[1], w[4]);
            w[6] = cmul(w[2], w[4]);
            w[7] = cmul(w[3], w[4]);
        }
#pragma unroll
        for (int r = 1; r < R; ++r) {
            float2 x = w[r];
            if constexpr (S > 0) x.y = -x.y;
            v[b * R + r] = cmul(v[b * R + r], x);
        }
        dft<R, S, b * R, 1>(v);
    });
}

// the same, with W^k, W^2k, W^4k (k < NS) read from shared rows at
// rows[k], rows[NS + k], rows[2 NS + k]
template <int M, int T, int R, int NS, int S, int P>
__device__ __forceinline__ void stage_compute_pow_rows(float2 (&v)[P], int t,
                                                       const float2* rows) {
    static_assert(R == 2 || R == 4 || R == 8, "power twiddles for radix 2, 4, 8");
    static_for<0, P / R>([&](auto Bb) {
        constexpr int b = decltype(Bb)::value;
        const int k = (t + T * b) % NS;
        float2 w[R];
        w[1] = rows[k];
        if constexpr (R >= 4) {
            w[2] = rows[NS + k];
            w[3] = cmul(w[1], w[2]);
        }
        if constexpr (R == 8) {
            w[4] = rows[2 * NS + k];
            w[5] = cmul(w[1], w[4]);
            w[6] = cmul(w[2], w[4]);
            w[7] = cmul(w[3], w[4]);
        }
#pragma unroll
        for (int r = 1; r < R; ++r) {
            float2 x = w[r];
            if constexpr (S > 0) x.y = -x.y;
            v[b * R + r] = cmul(v[b * R + r], x);
        }
        dft<R, S, b * R, 1>(v);
    });
}

// stages 2 and 3 after stage 1's DFT; the last stage's outputs (index
// n = j + r M / R_last, j = t + T b) go to `emit`
// (only the build switches that read the last stage's twiddles from global
// memory call it)
#pragma nv_diag_suppress 177
struct Tw2048 {
    const float2* w;
    __device__ __forceinline__ float2 operator()(int e) const { return __ldg(w + (e & 2047)); }
};
#pragma nv_diag_default 177

template <int M, int S, class Emit>
__device__ __forceinline__ void band_rest(float2 (&v)[kP], float2* buf, const float2* tws,
                                          const float2* bp_tw, int t, Emit emit) {
    constexpr int T = M / kP;
    using L = TwLayout<M>;
    constexpr int R1 = L::R1, R2 = L::R2, R3 = L::R3;
    using std::integral_constant;
    if constexpr (R2 == 1) {
        emit(v, integral_constant<int, R1>{}, integral_constant<int, 1>{});
    } else {
        stage_store<M, T, R1, 1, kSH>(v, buf, t);
        __syncthreads();
        stage_load<M, T, R2, kSH>(v, buf, t);
        __syncthreads();
        stage_compute_rows<M, T, R2, R1, S>(v, t, tws);
        if constexpr (R3 == 1) {
            emit(v, integral_constant<int, R2>{}, integral_constant<int, R1>{});
        } else {
            stage_store<M, T, R2, R1, kSH>(v, buf, t);
            __syncthreads();
            stage_load<M, T, R3, kSH>(v, buf, t);
            __syncthreads();
            if constexpr (FCQT_TW3_SMEM) {
                stage_compute_rows<M, T, R3, R1 * R2, S>(v, t, tws + L::n2);
            } else if constexpr (FCQT_TW_TMA) {
                stage_compute_pow_rows<M, T, R3, R1 * R2, S>(v, t, tws + L::n2);
            } else if constexpr (FCQT_TW3_POW) {
                stage_compute_pow<M, T, R3, R1 * R2, S, 2048>(v, t, Tw2048{bp_tw});
            } else {
                stage_compute<M, T, R3, R1 * R2, S, 2048>(v, t, Tw2048{bp_tw});
            }
            emit(v, integral_constant<int, R3>{}, integral_constant<int, R1 * R2>{});
        }
    }
}

__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
    const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(sa), "l"(gmem));
}

__device__ __forceinline__ void cp_async4(float* smem, const float* gmem) {
    const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(sa), "l"(gmem));
}

__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

// TMA bulk copies (no multicast): shared -> global stores tracked by a bulk
// group; the issuing thread waits only until shared memory has been read
__device__ __forceinline__ bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void bulk_store(void* gdst, const void* ssrc, unsigned bytes) {
    const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(ssrc));
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n"
                 ::"l"(gdst), "r"(sa), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_commit_wait_read() {
    asm volatile("cp.async.bulk.commit_group;\ncp.async.bulk.wait_group.read 0;\n" ::: "memory");
}

// TMA bulk loads completing on an mbarrier.  Every wait is bounded in time:
// a wait whose first poll fails reads the global nanosecond timer and gives
// up after kWaitLimitNs (a TMA bulk copy normally lands within microseconds),
// with kMaxWaitSpins polls as a second bound.  A wait that gives up counts
// itself in g_wait_timeouts (process-wide, cqt_wait_timeouts) and in the
// call's wait-status word (the workspace header, cqt_workspace_waits) and
// returns, so a lost completion can neither hang the GPU nor go unnoticed.
constexpr int kMaxWaitSpins = 1 << 22;
constexpr unsigned long long kWaitLimitNs = 1000000000ull;   // 1 s
__device__ unsigned int g_wait_timeouts;

__device__ __forceinline__ unsigned smem_u32(const void* p) {
    return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(unsigned long long* mbar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n"
                 "fence.mbarrier_init.release.cluster;\n"
                 ::"r"(smem_u32(mbar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect(unsigned long long* mbar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n"
                 ::"r"(smem_u32(mbar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_load(void* sdst, const void* gsrc, unsigned bytes,
                                          unsigned long long* mbar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1], %2, [%3];\n"
                 ::"r"(smem_u32(sdst)), "l"(gsrc), "r"(bytes), "r"(smem_u32(mbar)) : "memory");
}
__device__ __forceinline__ bool mbar_try(unsigned a, unsigned phase) {
    unsigned done;
    asm volatile("{\n.reg .pred p;\n"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                 "selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(done) : "r"(a), "r"(phase) : "memory");
    return done != 0;
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __noinline__ bool mbar_wait_slow(unsigned a, unsigned phase, unsigned* status) {
    const unsigned long long t0 = global_ns();
    for (int i = 0; i < kMaxWaitSpins; ++i) {
        if (mbar_try(a, phase)) return true;
        if (global_ns() - t0 > kWaitLimitNs) break;
    }
    atomicAdd(&g_wait_timeouts, 1u);
    if (status) atomicAdd(status, 1u);
    return false;
}
__device__ __forceinline__ bool mbar_wait(unsigned long long* mbar, unsigned phase,
                                          unsigned* status) {
    const unsigned a = smem_u32(mbar);
    if (mbar_try(a, phase)) return true;
    return mbar_wait_slow(a, phase, status);
}

// where an instance's M coefficients live: element n at
// base + ((n + roll) mod M) -- the per-slice heap (roll 0) or the sliced
// block layout (SliceLayout, roll +-M/4 on octave groups)
struct CoefAddr {
    long long base;
    int roll;
};

template <int M, bool SLICED>
__device__ __forceinline__ CoefAddr coef_addr(const BandParams& bp, int slice, int4 d) {
    CoefAddr a;
    if constexpr (!SLICED) {
        a.base = (long long)slice * bp.ncoef + d.x;
        a.roll = 0;
    } else {
        const int S = bp.sl.S;
        const long long row = slice / S;
        const int s = slice % S;
        const int gi = (d.w >> 12) & 15, r = (d.w >> 16) & 255;
        a.base = bp.sl.goff[gi] + ((row * bp.sl.grows[gi] + r) * S + s) * (long long)M;
        // roll parity follows the global slice index
        a.roll = bp.sl.groll[gi] ? (((bp.sl.slice0 + s) & 1) ? -(M / 4) : M / 4) : 0;
    }
    return a;
}

// descriptor fields: {heap offset, lo (octave) | band id (side), l | Lg << 16,
// flags: bit 0 side band, bits 4-7 synthesis plane, bits 8-11 adjoint plane}
__device__ __forceinline__ int d_l(int4 d) { return d.z & 0xFFFF; }
__device__ __forceinline__ int d_lg(int4 d) { return d.z >> 16; }
__device__ __forceinline__ int d_plane(int4 d, int which) { return (d.w >> (4 + 4 * which)) & 15; }

template <int M, bool SLICED, int KIND, bool EXT>
__device__ void band_fwd(const float2* __restrict__ X, const FwdTab& tab, const BandParams& bp,
                         int c, CoefPtr out, float2* smem, float2* tws,
                         unsigned long long* mbar) {
    constexpr int T = M / kP;
    constexpr int R1 = Sched<M>::R1;
    constexpr int IPC = kBandThreads / T;
    const Inst in = locate<M, EXT>(bp, c);
    const int t = in.t;
    float2* buf = smem + in.il * inst_stride(M);
    const float2* Xs = X + (long)in.slice * bp.stride;
    const int off = in.d.x;
    constexpr bool side = KIND == kSide;   // every instance of the class is of one kind
    // octave classes whose first-stage inputs r = 6..9 are outside every
    // band's window support (checked at upload) skip them: no gather, no
    // gain, a DFT that knows they are zero
    // (taps [6M/16, 10M/16): first-stage inputs 6..9 of a radix-16 butterfly,
    // 12..19 of a radix-32 one)
    constexpr unsigned kZero = KIND != kOctavePruned ? 0u : R1 == 16 ? 0x3C0u : 0xFF000u;
    static_assert(KIND != kOctavePruned || ((R1 == 16 || R1 == 32) && kP / R1 == 1),
                  "pruning assumes one radix-16 or radix-32 butterfly per thread in stage 1");

    // stage the band's contiguous spectrum segment [lo, lo + n), n <= M,
    // into shared memory with one TMA bulk load issued by the instance's
    // first thread: bins [lo & ~1, (lo + n + 1) & ~1) (16-byte aligned ends;
    // spectrum rows are 16-byte aligned and hold bins up to 32775), unpadded,
    // so bin lo + i sits at buf[i + (lo & 1)]
    int lo = 0, n = 0;
    if (in.valid) {
        if constexpr (side) {
            const int2 sg = __ldg(tab.seg + in.d.y);
            lo = sg.x;
            n = sg.y;
        } else {
            lo = in.d.y;
            n = d_lg(in.d);
        }
    }
    const int sh = lo & 1;
    if (threadIdx.x == 0) mbar_init(mbar, IPC);
    __syncthreads();
    pdl_wait();   // the previous kernel of the stream has completed
    if (t == 0) {
        const int a = lo - sh, bytes = n > 0 ? (((lo + n + 1) & ~1) - a) * 8 : 0;
        // the CTA's first thread also brings the twiddle slot
        const unsigned twb = (FCQT_TW_TMA && threadIdx.x == 0) ? TwSlot<M>::bytes : 0u;
        mbar_arrive_expect(mbar, (unsigned)bytes + twb + (bp.expire_waits ? 16u : 0u));
        if (bytes) bulk_load(buf, Xs + a, (unsigned)bytes, mbar);
        if (twb) bulk_load(tws, bp.twrows + tw_slot_index(M) * kBandTw, twb, mbar);
    }
    if constexpr (!FCQT_TW_TMA) fill_twiddles<M>(tws, bp.tw2048);
    // stage 1 taps: element r of butterfly b is tap t + T b + r M / R1.
    // Octave bands read segment entry (m + l) mod M inside the window
    // support; side bands go through the per-tap gather table (conjugated
    // mirror taps).  The barrier below is outside both branches: one CTA may
    // hold instances of both kinds.
    float gain[kP];
    int src[kP];
    const int l = d_l(in.d);
    {
        const float* gp = tab.gain + off + t;
#pragma unroll
        for (int b = 0; b < kP / R1; ++b)
#pragma unroll
            for (int r = 0; r < R1; ++r)
                gain[b * R1 + r] = (in.valid && !((kZero >> r) & 1u))
                                       ? __ldg(gp + T * b + r * (M / R1)) : 0.f;
    }
    if constexpr (side) {
        const int* sp = tab.src + off + t;
#pragma unroll
        for (int b = 0; b < kP / R1; ++b)
#pragma unroll
            for (int r = 0; r < R1; ++r) {
                const int sv = in.valid ? __ldg(sp + T * b + r * (M / R1)) : -1;
                src[b * R1 + r] = sv < 0 ? -1 : (((sv & 0xFFFF) - lo) | (sv & 0x10000));
            }
    }
    // each thread's completed wait makes the bulk-loaded segment visible to
    // it; the twiddle rows filled above are first read in stage 2, behind the
    // stage-1 exchange barrier, so no CTA barrier is needed here
    mbar_wait(mbar, 0, bp.status);
    float2 v[kP];
    const float2* seg = buf + sh;
    if constexpr (!side) {
#pragma unroll
        for (int b = 0; b < kP / R1; ++b)
#pragma unroll
            for (int r = 0; r < R1; ++r) {
                if ((kZero >> r) & 1u) {
                    v[b * R1 + r] = make_float2(0.f, 0.f);
                    continue;
                }
                const int i = (t + T * b + r * (M / R1) + l) & (M - 1);
                v[b * R1 + r] = i < n ? cscale(seg[i], gain[b * R1 + r])
                                      : make_float2(0.f, 0.f);
            }
    } else {
#pragma unroll
        for (int i = 0; i < kP; ++i) {
            const int sv = src[i];
            float2 val = make_float2(0.f, 0.f);
            if (sv >= 0) {
                float2 xv = seg[sv & 0xFFFF];
                if (sv & 0x10000) xv.y = -xv.y;
                val = cscale(xv, gain[i]);
            }
            v[i] = val;
        }
    }
    static_for<0, kP / R1>([&](auto Bb) {
        dftz<R1, +1, kZero, decltype(Bb)::value * R1, 1>(v);
    });
    __syncthreads();   // the staged segment is dead; stage 1 reuses the buffer

    const CoefAddr ca = coef_addr<M, SLICED>(bp, in.slice, in.d);
    const bool interleaved = out.interleaved != 0;   // uniform: hoisted out of the stores
    float2* og = reinterpret_cast<float2*>(out.re) + ca.base;
    float* ore = out.re + ca.base;
    float* oim = out.im + ca.base;
    // the instance's M outputs are gathered in shared memory in destination
    // order (roll applied) and leave as one TMA bulk store per array; a
    // destination that is not 16-byte aligned takes per-element stores
    const bool bulk = in.valid && (interleaved ? aligned16(og) : aligned16(ore) && aligned16(oim));
    band_rest<M, +1>(v, buf, tws, bp.tw2048, t, [&](float2 (&w)[kP], auto Rc, auto NSc) {
        constexpr int R = decltype(Rc)::value, NS = decltype(NSc)::value;
        if (!in.valid) return;
        if (bulk) {
            if (interleaved) {
#pragma unroll
                for (int b = 0; b < kP / R; ++b)
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const int nn = t + T * b + r * NS;
                        buf[SLICED ? ((nn + ca.roll) & (M - 1)) : nn] = w[b * R + r];
                    }
            } else {
                float* sre = reinterpret_cast<float*>(buf);
                float* sim = sre + M;
#pragma unroll
                for (int b = 0; b < kP / R; ++b)
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const int nn = t + T * b + r * NS;
                        const int ix = SLICED ? ((nn + ca.roll) & (M - 1)) : nn;
                        sre[ix] = w[b * R + r].x;
                        sim[ix] = w[b * R + r].y;
                    }
            }
        } else if (interleaved) {
#pragma unroll
            for (int b = 0; b < kP / R; ++b)
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int nn = t + T * b + r * NS;
                    og[SLICED ? ((nn + ca.roll) & (M - 1)) : nn] = w[b * R + r];
                }
        } else {
#pragma unroll
            for (int b = 0; b < kP / R; ++b)
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int nn = t + T * b + r * NS;
                    const int ix = SLICED ? ((nn + ca.roll) & (M - 1)) : nn;
                    ore[ix] = w[b * R + r].x;
                    oim[ix] = w[b * R + r].y;
                }
        }
    });
    // every thread's shared writes -> visible to the async proxy -> one
    // thread per instance issues the copies (the barrier is CTA-uniform)
    fence_proxy_async_smem();
    __syncthreads();
    if (bulk && t == 0) {
        if (interleaved) {
            bulk_store(og, buf, M * 8);
        } else {
            bulk_store(ore, buf, M * 4);
            bulk_store(oim, reinterpret_cast<float*>(buf) + M, M * 4);
        }
        bulk_commit_wait_read();   // shared memory stays live until read
    }
}

template <int M, bool SLICED, int KIND, bool EXT>
__device__ void band_inv(CoefPtr in_c, const InvTab& tab, int which, const BandParams& bp, int c,
                         float2* __restrict__ E, float2* smem, float2* tws,
                         unsigned long long* mbar) {
    constexpr int T = M / kP;
    constexpr int R1 = Sched<M>::R1;
    constexpr int IPC = kBandThreads / T;
    const Inst in = locate<M, EXT>(bp, c);
    const int t = in.t;
    float2* buf = smem + in.il * inst_stride(M);
    const int off = in.d.x;
    const CoefAddr ca = coef_addr<M, SLICED>(bp, in.slice, in.d);

    // stage the instance's M coefficients into shared memory, unpadded, in
    // tap order (roll undone): interleaved as float2[M], planar as float[M]
    // re then float[M] im.  One TMA bulk load per contiguous piece, issued by
    // the instance's first thread; unaligned sources take per-element copies.
    const bool interleaved = in_c.interleaved != 0;
    const float2* src2 = reinterpret_cast<const float2*>(in_c.re) + ca.base;
    const float* sre = in_c.re + ca.base;
    const float* sim = in_c.im + ca.base;
    const bool bulk = in.valid && (interleaved ? aligned16(src2) : aligned16(sre) && aligned16(sim));
    float* bre = reinterpret_cast<float*>(buf);
    float* bim = bre + M;
    if (threadIdx.x == 0) mbar_init(mbar, IPC);
    __syncthreads();
    pdl_wait();   // the previous kernel of the stream has completed
    if (t == 0) {
        // the CTA's first thread also brings the twiddle slot
        const unsigned twb = (FCQT_TW_TMA && threadIdx.x == 0) ? TwSlot<M>::bytes : 0u;
        mbar_arrive_expect(mbar, (bulk ? M * 8 : 0) + twb + (bp.expire_waits ? 16u : 0u));
        if (twb) bulk_load(tws, bp.twrows + tw_slot_index(M) * kBandTw, twb, mbar);
        if (bulk) {
            // smem [0, M - r) <- src [r, M), smem [M - r, M) <- src [0, r)
            const int r = SLICED ? (ca.roll & (M - 1)) : 0;
            if (interleaved) {
                bulk_load(buf, src2 + r, (M - r) * 8, mbar);
                if (r) bulk_load(buf + (M - r), src2, r * 8, mbar);
            } else {
                bulk_load(bre, sre + r, (M - r) * 4, mbar);
                bulk_load(bim, sim + r, (M - r) * 4, mbar);
                if (r) {
                    bulk_load(bre + (M - r), sre, r * 4, mbar);
                    bulk_load(bim + (M - r), sim, r * 4, mbar);
                }
            }
        }
    }
    if (in.valid && !bulk) {
#pragma unroll
        for (int k = 0; k < kP; ++k) {
            const int i = t + k * T;
            const int ix = SLICED ? ((i + ca.roll) & (M - 1)) : i;
            if (interleaved) {
                cp_async8(buf + i, src2 + ix);
            } else {
                cp_async4(bre + i, sre + ix);
                cp_async4(bim + i, sim + ix);
            }
        }
    }
    if constexpr (!FCQT_TW_TMA) fill_twiddles<M>(tws, bp.tw2048);
    cp_async_wait_all();
    mbar_wait(mbar, 0, bp.status);
    __syncthreads();
    float2 v[kP];
    if (interleaved) {
#pragma unroll
        for (int b = 0; b < kP / R1; ++b)
#pragma unroll
            for (int r = 0; r < R1; ++r) v[b * R1 + r] = buf[t + T * b + r * (M / R1)];
    } else {
#pragma unroll
        for (int b = 0; b < kP / R1; ++b)
#pragma unroll
            for (int r = 0; r < R1; ++r) {
                const int i = t + T * b + r * (M / R1);
                v[b * R1 + r] = make_float2(bre[i], bim[i]);
            }
    }
    if (!in.valid) {
#pragma unroll
        for (int i = 0; i < kP; ++i) v[i] = make_float2(0.f, 0.f);
    }
    static_for<0, kP / R1>([&](auto Bb) {
        dft<R1, -1, decltype(Bb)::value * R1, 1>(v);
    });
    __syncthreads();   // stage 1 reads done; the exchange reuses the buffer

    float2* Es = E + (long)in.slice * tab.nplanes * bp.stride;
    constexpr bool side = KIND == kSide;   // every instance of the class is of one kind
    const int lo = in.d.y, l = d_l(in.d), lg = d_lg(in.d);
    const int pbase = d_plane(in.d, which) * bp.stride + lo;
    // last-stage outputs r of a pruned octave class that lie outside every
    // band's window support (taps [6M/16, 10M/16), checked at upload): for
    // M = 2048 the radix-8 outputs 3 and 4 -- no gain, no index, no store
    constexpr int RL = TwLayout<M>::R3 > 1 ? TwLayout<M>::R3
                       : TwLayout<M>::R2 > 1 ? TwLayout<M>::R2 : TwLayout<M>::R1;
    constexpr unsigned kDeadOut = (KIND == kOctavePruned && M == 2048 && RL == 8) ? 0x18u : 0u;
#if FCQT_PREFETCH_GAINS
    // the gains of this thread's final-stage outputs, loaded before the
    // stages so the scatter does not wait on them
    constexpr int NSL = M / RL;
    float gpre[kP];
    if constexpr (!side) {
#pragma unroll
        for (int b = 0; b < kP / RL; ++b)
#pragma unroll
            for (int r = 0; r < RL; ++r)
                gpre[b * RL + r] = (in.valid && !((kDeadOut >> r) & 1u))
                                       ? __ldg(tab.gre + off + t + T * b + r * NSL) : 0.f;
    }
#endif
    band_rest<M, -1>(v, buf, tws, bp.tw2048, t, [&](float2 (&w)[kP], auto Rc, auto NSc) {
        constexpr int R = decltype(Rc)::value, NS = decltype(NSc)::value;
        if (!in.valid) return;
        if constexpr (side) {
#pragma unroll
            for (int b = 0; b < kP / R; ++b)
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int m = t + T * b + r * NS;
                    const float2 val = w[b * R + r];
                    const int d = __ldg(tab.dest + off + m);
                    if (d >= 0)
                        Es[d] = make_float2(val.x * __ldg(tab.gre + off + m),
                                            val.y * __ldg(tab.gim + off + m));
                }
        } else {
            float2* eb = Es + pbase;
#pragma unroll
            for (int b = 0; b < kP / R; ++b)
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    if ((kDeadOut >> r) & 1u) continue;
                    const int m = t + T * b + r * NS;
                    const int i = (m + l) & (M - 1);
#if FCQT_PREFETCH_GAINS
                    const float g = gpre[b * R + r];
#else
                    const float g = __ldg(tab.gre + off + m);
#endif
                    if (i < lg && g != 0.f) eb[i] = cscale(w[b * R + r], g);
                }
        }
    });
}

// class of this CTA: the number of class boundaries at or below blockIdx.x
// (branch-free; unused classes have cta0 == grid)
__device__ __forceinline__ int find_class(const BandSched& sc) {
    int c = 0;
#pragma unroll
    for (int k = 1; k < kMaxClasses; ++k)
        c += (k < sc.ncls && (int)blockIdx.x >= sc.cta0[k]) ? 1 : 0;
    return c;
}

template <bool SLICED, bool EXT>
__global__ void __launch_bounds__(kBandThreads, kBandMinBlocks)
bands_fwd_kernel(const float2* __restrict__ X, FwdTab tab, const __grid_constant__ BandParams bp,
                 CoefPtr out) {
    extern __shared__ float4 smem_raw[];
    __shared__ unsigned long long mbar;
    float2* smem = reinterpret_cast<float2*>(smem_raw);
    float2* tws = smem + kBandData;
    pdl_launch_dependents();
    const int c = find_class(bp.sc);
    const int kind = bp.sc.kind[c];
    auto run = [&](auto Mc) {
        constexpr int M = decltype(Mc)::value;
        if (kind == kSide)
            band_fwd<M, SLICED, kSide, EXT>(X, tab, bp, c, out, smem, tws, &mbar);
        else if (kind == kOctavePruned)
            band_fwd<M, SLICED, kOctavePruned, EXT>(X, tab, bp, c, out, smem, tws, &mbar);
        else
            band_fwd<M, SLICED, kOctave, EXT>(X, tab, bp, c, out, smem, tws, &mbar);
    };
    switch (bp.sc.M[c]) {
    case 2048: run(std::integral_constant<int, 2048>{}); break;
    case 1024: run(std::integral_constant<int, 1024>{}); break;
    case 512:  run(std::integral_constant<int, 512>{}); break;
    case 256:  run(std::integral_constant<int, 256>{}); break;
    case 128:  run(std::integral_constant<int, 128>{}); break;
    case 64:   run(std::integral_constant<int, 64>{}); break;
    case 32:   run(std::integral_constant<int, 32>{}); break;
    case 16:   if constexpr (kP <= 16) run(std::integral_constant<int, 16>{}); break;
    default: break;
    }
}

template <bool SLICED, bool EXT>
__global__ void __launch_bounds__(kBandThreads, kBandMinBlocks)
bands_inv_kernel(CoefPtr in, InvTab tab, int which, const __grid_constant__ BandParams bp,
                 float2* __restrict__ E) {
    extern __shared__ float4 smem_raw[];
    __shared__ unsigned long long mbar;
    float2* smem = reinterpret_cast<float2*>(smem_raw);
    float2* tws = smem + kBandData;
    pdl_launch_dependents();
    const int c = find_class(bp.sc);
    const bool side = bp.sc.kind[c] == kSide;
    const bool pruned = bp.sc.kind[c] == kOctavePruned;
    auto run = [&](auto Mc) {
        constexpr int M = decltype(Mc)::value;
        if (side)
            band_inv<M, SLICED, kSide, EXT>(in, tab, which, bp, c, E, smem, tws, &mbar);
        else if (M == 2048 && pruned)
            band_inv<M, SLICED, kOctavePruned, EXT>(in, tab, which, bp, c, E, smem, tws, &mbar);
        else
            band_inv<M, SLICED, kOctave, EXT>(in, tab, which, bp, c, E, smem, tws, &mbar);
    };
    switch (bp.sc.M[c]) {
    case 2048: run(std::integral_constant<int, 2048>{}); break;
    case 1024: run(std::integral_constant<int, 1024>{}); break;
    case 512:  run(std::integral_constant<int, 512>{}); break;
    case 256:  run(std::integral_constant<int, 256>{}); break;
    case 128:  run(std::integral_constant<int, 128>{}); break;
    case 64:   run(std::integral_constant<int, 64>{}); break;
    case 32:   run(std::integral_constant<int, 32>{}); break;
    case 16:   if constexpr (kP <= 16) run(std::integral_constant<int, 16>{}); break;
    default: break;
    }
}

}  // namespace

BandSched make_sched(int ncls, const int* M, const int* nb, const int* first, const int* kind,
                     int batch) {
    BandSched sc{};
    sc.ncls = ncls;
    sc.batch = batch;
    sc.inv_batch = batch > 0 ? 1.0f / (float)batch : 0.f;
    int cta = 0;
    for (int c = 0; c < ncls; ++c) {
        sc.M[c] = M[c];
        sc.nb[c] = nb[c];
        sc.first[c] = first[c];
        sc.kind[c] = kind[c];
        sc.cta0[c] = cta;
        const int ipc = kBandCap / M[c];
        const long inst = (long)nb[c] * batch;
        cta += (int)((inst + ipc - 1) / ipc);
    }
    sc.cta0[ncls] = cta;
    return sc;
}

cudaError_t launch_bands_fwd(const float2* X, const FwdTab& tab, const BandParams& bp,
                             CoefPtr out, cudaStream_t s) {
    const int grid = bp.sc.cta0[bp.sc.ncls];
    if (grid <= 0) return cudaSuccess;
    auto go = [&](auto kern) {
        return launch_pdl(bp.sc.batch <= kPdlMaxBatch, kern, dim3(grid), dim3(kBandThreads),
                          kBandSmem, s, X, tab, bp, out);
    };
    if (bp.sl.S > 0)
        return bp.ext ? go(bands_fwd_kernel<true, true>) : go(bands_fwd_kernel<true, false>);
    return bp.ext ? go(bands_fwd_kernel<false, true>) : go(bands_fwd_kernel<false, false>);
}

cudaError_t launch_bands_inv(CoefPtr in, const InvTab& tab, int which, const BandParams& bp,
                             float2* E, cudaStream_t s) {
    const int grid = bp.sc.cta0[bp.sc.ncls];
    if (grid <= 0) return cudaSuccess;
    auto go = [&](auto kern) {
        return launch_pdl(bp.sc.batch <= kPdlMaxBatch, kern, dim3(grid), dim3(kBandThreads),
                          kBandSmem, s, in, tab, which, bp, E);
    };
    if (bp.sl.S > 0)
        return bp.ext ? go(bands_inv_kernel<true, true>) : go(bands_inv_kernel<true, false>);
    return bp.ext ? go(bands_inv_kernel<false, true>) : go(bands_inv_kernel<false, false>);
}

namespace {
// one block length's slot: stage-2 rows W_{R1 R2}^{r k} (r = 1..R2-1, k < R1)
// as fill_twiddles gathers them, then the last stage's W^k, W^2k, W^4k
// (k < R1 R2) as stage_compute_pow reads them -- entries of W_2048 (host)
template <int M>
void slot_rows(float2* out, const float2* w2048) {
    using L = TwLayout<M>;
    using Sl = TwSlot<M>;
    for (int e = 0; e < L::n2; ++e) {
        const int r = e / L::R1 + 1, k = e % L::R1;
        out[e] = w2048[(r * k * (2048 / (L::R1 * L::R2))) & 2047];
    }
    const int scale3 = L::R3 > 1 ? 2048 / (Sl::NS3 * L::R3) : 0;
    for (int pi = 0; pi < Sl::npow; ++pi)
        for (int k = 0; k < Sl::NS3; ++k)
            out[L::n2 + pi * Sl::NS3 + k] = w2048[(((1 << pi) * k) * scale3) & 2047];
}
}  // namespace

int band_twiddle_count() { return kTwSlots * kBandTw; }

void band_twiddle_rows(float2* out, const float2* w2048) {
    for (int i = 0; i < kTwSlots * kBandTw; ++i) out[i] = make_float2(0.f, 0.f);
    if constexpr (!FCQT_TW_TMA) return;   // the kernels gather their twiddles
    if constexpr (kP <= 16) slot_rows<16>(out + tw_slot_index(16) * kBandTw, w2048);
    slot_rows<32>(out + tw_slot_index(32) * kBandTw, w2048);
    slot_rows<64>(out + tw_slot_index(64) * kBandTw, w2048);
    slot_rows<128>(out + tw_slot_index(128) * kBandTw, w2048);
    slot_rows<256>(out + tw_slot_index(256) * kBandTw, w2048);
    slot_rows<512>(out + tw_slot_index(512) * kBandTw, w2048);
    slot_rows<1024>(out + tw_slot_index(1024) * kBandTw, w2048);
    slot_rows<2048>(out + tw_slot_index(2048) * kBandTw, w2048);
}

cudaError_t read_wait_timeouts(unsigned* count) {
    return cudaMemcpyFromSymbol(count, g_wait_timeouts, sizeof(unsigned));
}

cudaError_t init_band_attributes() {
    const void* fns[] = {(const void*)bands_fwd_kernel<false, false>,
                         (const void*)bands_fwd_kernel<true, false>,
                         (const void*)bands_inv_kernel<false, false>,
                         (const void*)bands_inv_kernel<true, false>,
                         (const void*)bands_fwd_kernel<false, true>,
                         (const void*)bands_fwd_kernel<true, true>,
                         (const void*)bands_inv_kernel<false, true>,
                         (const void*)bands_inv_kernel<true, true>};
    for (const void* f : fns) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kBandSmem);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace fcqt
