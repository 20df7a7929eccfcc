// Packed real-FFT engine: x (65536 real samples per slice) <-> X (32769-bin
// half spectrum), the front end of the analysis and the back end of the
// synthesis.
//
// The 65536-point real FFT is computed as the 32768-point complex FFT of
// z[n] = x[2n] + i x[2n+1] (the reference's packing, packedfft.cu:1-6), split
// radix-2 across the two CTAs of a slice:
//   CTA 0 transforms u0[n] = z[n] + z[n + 16384]               -> Z[2k]
//   CTA 1 transforms u1[n] = (z[n] - z[n + 16384]) W_32768^n   -> Z[2k + 1]
// so each CTA holds a 16384-point problem (132 KB with padding) entirely in
// shared memory and runs it as Stockham stages (32 x 32 x 16 with 512
// threads of 32 points for the forward, 16 x 16 x 16 x 4 with 1024 threads of
// 16 points for the inverse -- the faster schedule of each on B200),
// then untangles the (q, L - q) bin pairs of its parity -- which are all
// local -- into the real spectrum X[q] (spectral recovery of fused.py:311-328,
// done once per bin instead of once per router tap).
// The inverse mirrors it: each CTA rebuilds the packed spectrum from the
// colour planes on the fly (quads {n, 16384 - n, 16384 + n, 32768 - n} close
// under both the retangle and the DIF maps), forms its DIF half, runs the
// inverse Stockham stages and stores z[2m + h] de-interleaved into y.
//
// Stage twiddles W_{NS R}^{r k} come from shared rows that every warp reads
// without bank conflicts: direct rows [r][k] for spans NS <= 32, and for
// larger spans a split W^{r k} = lo[r][k mod 32] * hi[r][k / 32] (lo rows are
// read lane-consecutive, hi rows are warp-uniform broadcasts).  The library
// generates the rows in double precision at table upload.
#include <cmath>
#include <cstdint>
#include <type_traits>

#include <cooperative_groups.h>

// the spectrum kernels keep scalar complex adds: the packed two-lane form
// measured about 1 % slower here (it is faster in the band kernels)
#ifndef FCQT_F32X2
#define FCQT_F32X2 0
#endif

#include "engine.cuh"
#include "internal.h"

namespace fcqt {

// points per thread of the forward and inverse kernels (16 -> 1024 threads,
// stages 16 x 16 x 16 x 4; 32 -> 512 threads, stages 32 x 32 x 16)
#ifndef FCQT_SPEC_P_FWD
#define FCQT_SPEC_P_FWD 32
#endif
#ifndef FCQT_SPEC_P_INV
#define FCQT_SPEC_P_INV 16
#endif

namespace {

// a Stockham schedule: transform length N, P points per thread (T = N / P
// threads), NST stages of radices R1..R4
template <int N_, int P_, int NST_, int R1_, int R2_, int R3_, int R4_>
struct SpecSched {
    static constexpr int N = N_, P = P_, T = N_ / P_, NST = NST_;
    static constexpr int R1 = R1_, R2 = R2_, R3 = R3_, R4 = R4_;
};
// 16384 points per CTA (two CTAs per slice, one CTA per SM)
using S16k32 = SpecSched<16384, 32, 3, 32, 32, 16, 1>;
using S16k16 = SpecSched<16384, 16, 4, 16, 16, 16, 4>;
// 8192 points per CTA: 32768-sample slices
using S8k32 = SpecSched<8192, 32, 3, 32, 16, 16, 1>;
using S8k16 = SpecSched<8192, 16, 4, 16, 16, 16, 2>;

template <class C>
constexpr int sR(int s) { return s == 1 ? C::R1 : s == 2 ? C::R2 : s == 3 ? C::R3 : C::R4; }
template <class C>
constexpr int sNS(int s) { return s <= 1 ? 1 : sNS<C>(s - 1) * sR<C>(s - 1); }
template <class C>
constexpr bool sSplit(int s) { return sNS<C>(s) > 32; }
template <class C>
constexpr int sSize(int s) {
    return (s < 2 || s > C::NST) ? 0
           : sSplit<C>(s) ? sR<C>(s) * 32 + sR<C>(s) * (sNS<C>(s) / 32)
                          : (sR<C>(s) - 1) * sNS<C>(s);
}
template <class C>
constexpr int sOff(int s) { return s <= 2 ? 0 : sOff<C>(s - 1) + sSize<C>(s - 1); }
template <class C>
constexpr int twTotal() { return sOff<C>(C::NST + 1); }
template <class C>
constexpr int shiftOf() { return C::P == 32 ? 5 : 4; }   // shared padding shift
template <class C>
constexpr int smemOf() { return (padded<shiftOf<C>()>(C::N) + 512 + twTotal<C>()) * 8; }

template <class C>
constexpr bool sched_ok() { return sNS<C>(C::NST) * sR<C>(C::NST) == C::N; }
static_assert(sched_ok<S16k32>() && sched_ok<S16k16>() && sched_ok<S8k32>() && sched_ok<S8k16>(),
              "stage radices must multiply to the length");

// the twiddle-row blob holds the rows of every schedule, in this order
template <class C>
constexpr int rowsOff() {
    return std::is_same<C, S16k32>::value   ? 0
           : std::is_same<C, S16k16>::value ? twTotal<S16k32>()
           : std::is_same<C, S8k32>::value  ? twTotal<S16k32>() + twTotal<S16k16>()
                                            : twTotal<S16k32>() + twTotal<S16k16>() +
                                                  twTotal<S8k32>();
}
constexpr int kSpecRowsTotal =
    twTotal<S16k32>() + twTotal<S16k16>() + twTotal<S8k32>() + twTotal<S8k16>();

// the slice geometry: N samples, L = N/2 packed complex points, Q = N/4 per
// CTA, spectrum rows / colour planes of STRIDE complex values, and W_N^e =
// W_65536^(e TWM) from the shared two-level W_65536 table
template <int NS>
struct Geo {
    static constexpr int N = NS, L = NS / 2, Q = NS / 4, STRIDE = NS / 2 + 8,
                         TWM = 65536 / NS;
    static_assert(NS == 65536 || NS == 32768, "slices of 65536 or 32768 samples");
};
// forward / inverse schedule of each geometry
template <class G>
using CFg = typename std::conditional<
    G::N == 65536, std::conditional<FCQT_SPEC_P_FWD == 32, S16k32, S16k16>::type,
    std::conditional<FCQT_SPEC_P_FWD == 32, S8k32, S8k16>::type>::type;
template <class G>
using CIg = typename std::conditional<
    G::N == 65536, std::conditional<FCQT_SPEC_P_INV == 32, S16k32, S16k16>::type,
    std::conditional<FCQT_SPEC_P_INV == 32, S8k32, S8k16>::type>::type;

struct Tw64k {
    const float2* hi;
    const float2* lo;
    __device__ __forceinline__ float2 operator()(int e) const { return tw64k(hi, lo, e); }
};

// the two-level W_65536 tables and the stage rows of schedule C, staged by
// asynchronous copies (16 bytes each, no register round trip): issued at
// kernel start, so that they arrive while the CTA's first global loads are in
// flight; each thread waits for its own copies (cp_async_wait_all), and a CTA
// barrier then publishes everyone's
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
}

template <class C, int NT = C::T>
__device__ __forceinline__ void load_tables_async(float2* sm_hilo, float2* sm_tw,
                                                  const float2* ghi, const float2* glo,
                                                  const float2* gtw) {
    static_assert(rowsOff<C>() % 2 == 0 && twTotal<C>() % 2 == 0, "16-byte copies");
    gtw += rowsOff<C>();
    constexpr int kChunks = (512 + twTotal<C>()) / 2;
    for (int i = threadIdx.x; i < kChunks; i += NT) {
        const int e = 2 * i;
        const float2* src = e < 256 ? ghi + e : e < 512 ? glo + (e - 256) : gtw + (e - 512);
        float2* dst = e < 512 ? sm_hilo + e : sm_tw + (e - 512);
        cp_async16(dst, src);
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}

// twiddle and DFT of stage s (all butterflies of the thread)
template <class C, int s, int S>
__device__ __forceinline__ void spec_compute(float2 (&v)[C::P], int t, const float2* tws) {
    constexpr int R = sR<C>(s), NS = sNS<C>(s), off = sOff<C>(s);
    constexpr int T = C::T;
    static_for<0, C::P / R>([&](auto Bb) {
        constexpr int b = decltype(Bb)::value;
        if constexpr (s > 1) {
            const int k = (t + T * b) % NS;
#pragma unroll
            for (int r = 1; r < R; ++r) {
                float2 w;
                if constexpr (sSplit<C>(s)) {
                    w = cmul(tws[off + r * 32 + (k & 31)],
                             tws[off + R * 32 + r * (NS / 32) + (k >> 5)]);
                } else {
                    w = tws[off + (r - 1) * NS + k];
                }
                if constexpr (S > 0) w.y = -w.y;
                v[b * R + r] = cmul(v[b * R + r], w);
            }
        }
        dft<R, S, b * R, 1>(v);
    });
}

// stages s..NST (stage s - 1 is computed and held in v); `fin` receives the
// last stage's outputs, index n = j + r NS_last for j = t + T b
template <class C, int s, int S, class Fin>
__device__ __forceinline__ void spec_stages(float2 (&v)[C::P], float2* buf, const float2* tws,
                                            int t, Fin fin) {
    constexpr int T = C::T, SH = shiftOf<C>();
    if constexpr (s > C::NST) {
        fin(v);
    } else {
        stage_store<C::N, T, sR<C>(s - 1), sNS<C>(s - 1), SH>(v, buf, t);
        __syncthreads();
        stage_load<C::N, T, sR<C>(s), SH>(v, buf, t);
        __syncthreads();
        spec_compute<C, s, S>(v, t, tws);
        spec_stages<C, s + 1, S>(v, buf, tws, t, fin);
    }
}

// one packed input pair z[n] = (sample 2n, sample 2n + 1) of slice g
struct SliceReader {
    const float* at;       // sliced: row element of slice position 0 (may lie
                           // outside the row; only [jl, jh) is read); else the slice
    int jl, jh;            // readable slice positions [jl, jh) (sliced)
    int shift;             // +-H
    int nmask;             // slice samples - 1
    const float* window;
    bool sliced;
    bool whole;            // sliced, every position readable, row and window
                           // 8-byte aligned at even positions: float2 loads
    __device__ __forceinline__ float2 operator()(int n) const {
        if (!sliced) return __ldg(reinterpret_cast<const float2*>(at) + n);
        const int j = (2 * n + shift) & nmask;
        float2 v;
        v.x = (j >= jl && j < jh) ? __ldg(at + j) : 0.f;
        v.y = (j + 1 >= jl && j + 1 < jh) ? __ldg(at + j + 1) : 0.f;
        if (window) {
            v.x *= __ldg(window + j);
            v.y *= __ldg(window + j + 1);
        }
        return v;
    }
    // the same value when `whole` holds
    __device__ __forceinline__ float2 pair(int n) const {
        const int j = (2 * n + shift) & nmask;
        float2 v = __ldg(reinterpret_cast<const float2*>(at + j));
        if (window) {
            const float2 w = __ldg(reinterpret_cast<const float2*>(window + j));
            v.x *= w.x;
            v.y *= w.y;
        }
        return v;
    }
};

// a float row indexed by global sample (row base - sample0) and the window
// both 8-byte aligned, so that even global samples start float2 pairs
__device__ __forceinline__ bool pairs_aligned(const float* row, long long sample0,
                                              const float* window) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(row) - (uintptr_t)(sample0 * 4);
    return ((a | reinterpret_cast<uintptr_t>(window)) & 7u) == 0;
}

// global sample range a buffer row can hold: [max(0, sample0), min(length, sample0 + count))
__device__ __forceinline__ void sample_range(const SigMap& m, long long& lo, long long& hi) {
    lo = m.sample0 > 0 ? m.sample0 : 0;
    hi = m.sample0 + m.count < m.length ? m.sample0 + m.count : m.length;
}

template <class G>
__device__ __forceinline__ int clamp_slice(long long v) {
    return v < 0 ? 0 : (v > G::N ? G::N : (int)v);
}

template <bool SLICED, class G>
__device__ __forceinline__ SliceReader make_reader(const SigMap& m, long long g) {
    SliceReader r;
    r.sliced = SLICED;
    r.window = m.window;
    r.whole = false;
    r.nmask = G::N - 1;
    if constexpr (!SLICED) {
        r.at = m.x + g * G::N;
        r.jl = r.jh = 0;
        r.shift = 0;
    } else {
        const long long row = g / m.S;
        const int sg = m.slice0 + (int)(g % m.S);
        const float* rp = m.x + row * m.ld;
        const long long p0 = 2LL * G::Q * (sg - 1);   // global sample of position 0
        long long lo, hi;
        sample_range(m, lo, hi);
        r.jl = clamp_slice<G>(lo - p0);
        r.jh = clamp_slice<G>(hi - p0);
        r.at = rp + (p0 - m.sample0);
        r.shift = (sg & 1) ? -G::Q : G::Q;
        r.whole = r.jl == 0 && r.jh == G::N && pairs_aligned(rp, m.sample0, r.window);
    }
    return r;
}

// L2 prefetch of one 128-byte line
__device__ __forceinline__ void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}
// bulk L2 prefetch (TMA, no multicast) of a 16-byte aligned range, in 64 KB
// pieces issued by threads 0, 1, ...; p and bytes multiples of 16
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, long long bytes, int t) {
    constexpr long long kPiece = 65536;
    const long long at = (long long)t * kPiece;
    if (at < bytes) {
        const long long n = bytes - at < kPiece ? bytes - at : kPiece;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(
                         static_cast<const char*>(p) + at), "r"((unsigned)n) : "memory");
    }
}

// Each spectrum CTA holds a whole SM (one CTA per SM), and the CTAs of a wave
// move in step: all load, then all compute while HBM idles.  So once a CTA
// has its own input it prefetches into L2 the input of the CTA one wave
// ahead (`ahead` = the number of resident CTAs), overlapping that HBM traffic
// with its compute; the next wave then loads at L2 speed.  Only addresses
// inside the readable ranges are touched.
template <bool SLICED, int T, class G>
__device__ __forceinline__ void prefetch_signal_part(const SigMap& m, long g, int part, int parts,
                                                     int t) {
    const int len = G::N / parts;
    if constexpr (!SLICED) {
        const float* base = m.x + g * G::N + part * len;
        if ((reinterpret_cast<uintptr_t>(base) & 15u) == 0) {
            prefetch_l2_bulk(base, (long long)len * 4, t);
        } else {   // 8-byte aligned signal: per-line prefetches
            for (int i = t; i < len / 32; i += T) prefetch_l2(base + 32 * i);
        }
    } else {
        const long long row = g / m.S;
        const int sg = m.slice0 + (int)(g % m.S);
        long long lo, hi;
        lo = m.sample0 > 0 ? m.sample0 : 0;
        hi = m.sample0 + m.count < m.length ? m.sample0 + m.count : m.length;
        long long a = 2LL * G::Q * (sg - 1) + (long long)part * len;
        long long b = a + len;
        a = a > lo ? a : lo;
        b = b < hi ? b : hi;
        if (a >= b) return;
        const float* r = m.x + row * m.ld - m.sample0;
        const int lines = (int)((b - a + 31) / 32);
        for (int i = t; i < lines; i += T) {
            const long long p = a + 32LL * i;
            prefetch_l2(r + (p < b ? p : b - 1));
        }
    }
}

template <int MODE, class G>
__global__ void __launch_bounds__(CFg<G>::T, 1)
spectrum_fwd_kernel(const SigMap in, float2* __restrict__ X,
                    const float2* __restrict__ ghi, const float2* __restrict__ glo,
                    const float2* __restrict__ gtw, int ahead) {
    using C = CFg<G>;
    constexpr int kHalf = G::L, kQuarter = G::Q, kPlaneStride = G::STRIDE;
    constexpr bool SLICED = MODE == kSigSliced;
    constexpr int P = C::P, T = C::T, SH = shiftOf<C>();
    extern __shared__ float4 smem_raw[];
    float2* buf = reinterpret_cast<float2*>(smem_raw);
    float2* hl = buf + padded<SH>(kQuarter);
    float2* tws = hl + 512;
    const int h = blockIdx.x & 1;
    const long slice = blockIdx.x >> 1;
    const int t = threadIdx.x;
    pdl_launch_dependents();
    load_tables_async<C>(hl, tws, ghi, glo, gtw);
    pdl_wait();   // the previous kernel of the stream has completed
    const Tw64k tw{hl, hl + 256};

    // stage 1 inputs straight from global: the radix-2 DIF split of z (the
    // odd half's twiddles once the tables have landed)
    const SliceReader z = make_reader<SLICED, G>(in, slice);
    float2 v[P];
    auto load = [&](auto&& zf) {
#pragma unroll
        for (int b = 0; b < P / C::R1; ++b)
#pragma unroll
            for (int r = 0; r < C::R1; ++r) {
                const int n = t + T * b + r * (kQuarter / C::R1);
                const float2 a = zf(n);
                const float2 c = zf(n + kQuarter);
                v[b * C::R1 + r] = h == 0 ? cadd(a, c) : csub(a, c);
            }
        cp_async_wait_all();
        __syncthreads();
        if (h) {
#pragma unroll
            for (int b = 0; b < P / C::R1; ++b)
#pragma unroll
                for (int r = 0; r < C::R1; ++r) {
                    const int n = t + T * b + r * (kQuarter / C::R1);
                    v[b * C::R1 + r] = cmul(v[b * C::R1 + r], tw(2 * n * G::TWM));
                }
        }
    };
    if constexpr (MODE == kSigSqErr) {
        // the MSE gradient s (y - target) formed on load (s = 2 dL/dloss / n)
        const float2* yp = reinterpret_cast<const float2*>(in.x) + slice * (long)kHalf;
        const float2* tp = reinterpret_cast<const float2*>(in.target) + slice * (long)kHalf;
        const float sc = in.scale_dev ? in.scale * __ldg(in.scale_dev) : in.scale;
        load([&](int n) {
            const float2 a = __ldg(yp + n), b = __ldg(tp + n);
            return make_float2(sc * (a.x - b.x), sc * (a.y - b.y));
        });
    } else if (SLICED && z.whole) {   // one uniform branch, each side a straight run of loads
        load([&](int n) { return z.pair(n); });
    } else {
        load(z);
    }
    spec_compute<C, 1, -1>(v, t, tws);   // consumes the loads
    if (ahead > 0 && blockIdx.x + ahead < gridDim.x) {
        const long nb = blockIdx.x + (long)ahead;
        prefetch_signal_part<SLICED, T, G>(in, nb >> 1, (int)(nb & 1), 2, t);
        if constexpr (MODE == kSigSqErr) {
            SigMap tm = in;
            tm.x = in.target;
            prefetch_signal_part<false, T, G>(tm, nb >> 1, (int)(nb & 1), 2, t);
        }
    }
    spec_stages<C, 2, -1>(v, buf, tws, t, [&](float2 (&w)[P]) {
        stage_store<kQuarter, T, sR<C>(C::NST), sNS<C>(C::NST), SH>(w, buf, t);
    });
    __syncthreads();

    // untangle the (q, L - q) pairs of this parity: X[q] = E + W_N^q O
    // (natural bin order; the partner CTA writes the other parity)
    float2* Xs = X + slice * kPlaneStride;
    const int npairs = h == 0 ? kQuarter / 2 + 1 : kQuarter / 2;
    constexpr int NPIT = (kQuarter / 2 + 1 + T - 1) / T;
#pragma unroll
    for (int it = 0; it < NPIT; ++it) {
        const int kp = t + it * T;
        if (kp >= npairs) break;
        const int kq = h == 0 ? ((kQuarter - kp) & (kQuarter - 1)) : (kQuarter - 1 - kp);
        const float2 zq = buf[PADI<SH>(kp)];
        const float2 zb = buf[PADI<SH>(kq)];
        const int q = 2 * kp + h;
        const float2 w = tw(q * G::TWM);
        const float2 sq = cadd(zq, cconj(zb));
        const float2 dq = csub(zq, cconj(zb));
        const float2 wd = cmul(w, dq);
        // X[q] = (sq - i W^q dq) / 2
        Xs[q] = make_float2(0.5f * (sq.x + wd.y), 0.5f * (sq.y - wd.x));
        if (kq != kp || q == 0) {
            // X[L - q] = (conj(sq) + i conj(W^q) (-conj(dq))) / 2
            const float2 sb = cconj(sq);
            const float2 db = make_float2(-dq.x, dq.y);
            const float2 wdb = cmulc(db, w);
            Xs[kHalf - q] = make_float2(0.5f * (sb.x - wdb.y), 0.5f * (sb.y + wdb.x));
        }
    }
}

// F[q] from the colour planes flagged in the 4-bit mask mk, fixed plane order.
// Planes 0 and 1 cover almost every bin, so they are loaded unconditionally
// (e0, e1, in parallel with the mask) and selected; planes 2 and 3 are rare.
template <int STRIDE>
__device__ __forceinline__ float2 plane_pick(const float2* __restrict__ Es, unsigned mk, int q,
                                             float2 e0, float2 e1) {
    float2 acc = make_float2(0.f, 0.f);
    if (mk & 1u) acc = cadd(acc, e0);
    if (mk & 2u) acc = cadd(acc, e1);
    if (mk & 4u) acc = cadd(acc, Es[2 * STRIDE + q]);
    if (mk & 8u) acc = cadd(acc, Es[3 * STRIDE + q]);
    return acc;
}

// packed spectrum Zs[q] = E + i O, E = (a + conj b)/2, O = (a - conj b) W_N^-q / 2
__device__ __forceinline__ float2 retangle(float2 a, float2 b, float2 wq) {
    const float2 e = make_float2(0.5f * (a.x + b.x), 0.5f * (a.y - b.y));
    const float2 d = make_float2(0.5f * (a.x - b.x), 0.5f * (a.y + b.y));
    const float2 o = cmulc(d, wq);
    return make_float2(e.x - o.y, e.y + o.x);
}

// The two CTAs of a slice form a cluster.  Each rebuilds half of the quads
// {n, L - n, Q + n, Q - n} (four bins in; u_0 and u_1 at n and Q - n out)
// and writes the partner's half-spectrum values straight into the partner's
// shared memory, so every plane value is loaded once.  After that exchange
// the CTAs work alone: CTA h stores z[2m + h] into y (swapping halves through
// distributed shared memory for whole-sector stores measured slower).
template <int MODE, class G>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(CIg<G>::T, 1)
spectrum_inv_kernel(const float2* __restrict__ E, const unsigned short* __restrict__ qmask,
                    const SigMap out, const float2* __restrict__ ghi,
                    const float2* __restrict__ glo, const float2* __restrict__ gtw,
                    int nplanes, int ahead) {
    using C = CIg<G>;
    constexpr int kSlice = G::N, kHalf = G::L, kQuarter = G::Q, kPlaneStride = G::STRIDE;
    constexpr int P = C::P, T = C::T, SH = shiftOf<C>();
    namespace cg = cooperative_groups;
    extern __shared__ float4 smem_raw[];
    float2* buf = reinterpret_cast<float2*>(smem_raw);
    float2* hl = buf + padded<SH>(kQuarter);
    float2* tws = hl + 512;
    cg::cluster_group cl = cg::this_cluster();
    const int h = (int)cl.block_rank();
    float2* peer = cl.map_shared_rank(buf, h ^ 1);
    const long slice = blockIdx.x >> 1;
    const int t = threadIdx.x;
    pdl_launch_dependents();
    load_tables_async<C>(hl, tws, ghi, glo, gtw);
    cl.sync();   // the partner is running (its buffer may be written)
    pdl_wait();  // the previous kernel of the stream has completed
    const Tw64k tw{hl, hl + 256};
    const float2* Es = E + slice * (long)(nplanes * kPlaneStride);
    const bool two = nplanes > 1;

    // quads n in [0, Q/4) on CTA 0, [Q/4, Q/2] on CTA 1
    const int nlo = h ? kQuarter / 4 : 0;
    const int nhi = h ? kQuarter / 2 + 1 : kQuarter / 4;
    float2* u0 = h ? peer : buf;   // receives u_0
    float2* u1 = h ? buf : peer;   // receives u_1
    // software-pipelined by hand: the next quad's plane values are loaded
    // before this quad's shared-memory stores (the compiler may not move
    // global loads across stores through generic pointers)
    struct QuadIn {
        unsigned qm;
        float2 a0, b0, c0, d0, a1, b1, c1, d1;
    };
    auto load_quad = [&](int n) {
        QuadIn q;
        const float2 zero = make_float2(0.f, 0.f);
        q.qm = __ldg(qmask + n);
        q.a0 = Es[n];
        q.b0 = Es[kHalf - n];
        q.c0 = Es[kQuarter + n];
        q.d0 = Es[kQuarter - n];
        q.a1 = two ? Es[kPlaneStride + n] : zero;
        q.b1 = two ? Es[kPlaneStride + kHalf - n] : zero;
        q.c1 = two ? Es[kPlaneStride + kQuarter + n] : zero;
        q.d1 = two ? Es[kPlaneStride + kQuarter - n] : zero;
        return q;
    };
    int n = nlo + t;
    QuadIn cur;
    if (n < nhi) cur = load_quad(n);
    cp_async_wait_all();   // the tables have landed (own copies; the barrier: all)
    __syncthreads();
    for (; n < nhi; n += T) {
        QuadIn nxt;
        if (n + T < nhi) nxt = load_quad(n + T);
        const int bA = n, bB = kHalf - n, bC = kQuarter + n, bD = kQuarter - n;
        const unsigned qm = cur.qm;
        float2 fA = plane_pick<kPlaneStride>(Es, qm & 15u, bA, cur.a0, cur.a1);
        float2 fB = plane_pick<kPlaneStride>(Es, (qm >> 4) & 15u, bB, cur.b0, cur.b1);
        const float2 fC = plane_pick<kPlaneStride>(Es, (qm >> 8) & 15u, bC, cur.c0, cur.c1);
        const float2 fD = plane_pick<kPlaneStride>(Es, qm >> 12, bD, cur.d0, cur.d1);
        if (n == 0) {  // irfft ignores the imaginary parts of DC and Nyquist
            fA.y = 0.f;
            fB.y = 0.f;
        }
        // every twiddle of the quad follows from W^n and W^2n exactly
        // (W = W_65536, W^Q = -i): W^{Q+n} = -i W^n, W^{Q-n} = -i conj(W^n),
        // W^{2Q-n} = -conj(W^n), W^{2Q-2n} = -conj(W^2n)
        const float2 wn = tw(n * G::TWM);
        const float2 w2n = tw(2 * n * G::TWM);
        const float2 z0 = retangle(fA, fB, wn);
        const float2 z1 = retangle(fC, fD, make_float2(wn.y, -wn.x));
        u0[PADI<SH>(n)] = cadd(z0, z1);
        u1[PADI<SH>(n)] = cmulc(csub(z0, z1), w2n);
        const int m = kQuarter - n;
        if (m != n && m < kQuarter) {
            const float2 z2 = retangle(fD, fC, make_float2(-wn.y, -wn.x));
            const float2 z3 = retangle(fB, fA, make_float2(-wn.x, wn.y));
            u0[PADI<SH>(m)] = cadd(z2, z3);
            u1[PADI<SH>(m)] = cmulc(csub(z2, z3), make_float2(-w2n.x, w2n.y));
        }
        cur = nxt;
    }
    if (ahead > 0 && blockIdx.x + ahead < gridDim.x) {
        // planes 0 and 1 (read unconditionally) of the slice one wave ahead:
        // CTA h of that pair prefetches plane h (rows are 16-byte aligned)
        const long nb = blockIdx.x + (long)ahead;
        const int pl = (int)(nb & 1);
        if (pl < nplanes)
            prefetch_l2_bulk(E + (nb >> 1) * (long)(nplanes * kPlaneStride) +
                                 (long)pl * kPlaneStride,
                             (long long)kPlaneStride * 8, t);
    }
    cl.sync();   // both halves of u_h are in place

    float2 v[P];
    stage_load<kQuarter, T, C::R1, SH>(v, buf, t);
    __syncthreads();
    spec_compute<C, 1, +1>(v, t, tws);
    const float inv = 1.0f / (float)kHalf;
    if constexpr (MODE == kSigPlain) {
        // z[2m + h] -> samples 4m + 2h, 4m + 2h + 1
        float2* ys = reinterpret_cast<float2*>(out.y + slice * kSlice);
        spec_stages<C, 2, +1>(v, buf, tws, t, [&](float2 (&w)[P]) {
            constexpr int R = sR<C>(C::NST), NS = sNS<C>(C::NST);
#pragma unroll
            for (int b = 0; b < P / R; ++b)
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int nn = t + T * b + NS * r;
                    ys[2 * nn + h] = cscale(w[b * R + r], inv);
                }
        });
    } else if constexpr (MODE == kSigSqErr) {
        // the same stores, and the squared error against the target summed
        // in a fixed order: per thread, then a warp butterfly, then the warps
        // in index order -> one partial per CTA
        float2* ys = reinterpret_cast<float2*>(out.y + slice * kSlice);
        const float2* ts = reinterpret_cast<const float2*>(out.target + slice * kSlice);
        float acc = 0.f;
        spec_stages<C, 2, +1>(v, buf, tws, t, [&](float2 (&w)[P]) {
            constexpr int R = sR<C>(C::NST), NS = sNS<C>(C::NST);
#pragma unroll
            for (int b = 0; b < P / R; ++b)
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int nn = t + T * b + NS * r;
                    const float2 val = cscale(w[b * R + r], inv);
                    ys[2 * nn + h] = val;
                    const float2 tv = __ldg(ts + 2 * nn + h);
                    const float dx = val.x - tv.x, dy = val.y - tv.y;
                    acc = fmaf(dx, dx, acc);
                    acc = fmaf(dy, dy, acc);
                }
        });
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
        __shared__ float warp_sum[T / 32];
        if ((t & 31) == 0) warp_sum[t >> 5] = acc;
        __syncthreads();
        if (t == 0) {
            float sum = 0.f;
            for (int w = 0; w < T / 32; ++w) sum += warp_sum[w];
            out.partial[blockIdx.x] = sum;
        }
    } else {
        // un-roll by +-H and overlap-add into the zeroed output: every output
        // sample receives exactly two terms, and a + b == b + a, so the
        // result does not depend on the order of the two atomic adds
        const long long row = slice / out.S;
        const int sg = out.slice0 + (int)(slice % out.S);
        float* yr = out.y + row * out.ld - out.sample0;   // indexed by global sample
        const long long p0 = 2LL * kQuarter * (sg - 1);
        const int shift = (sg & 1) ? -kQuarter : kQuarter;
        const float* wnd = out.window;
        long long lo, hi;
        sample_range(out, lo, hi);
        // aligned rows take one two-lane vector atomic per pair (each lane
        // still receives exactly two terms)
        const bool vec = pairs_aligned(out.y + row * out.ld, out.sample0, wnd);
        spec_stages<C, 2, +1>(v, buf, tws, t, [&](float2 (&w)[P]) {
            constexpr int R = sR<C>(C::NST), NS = sNS<C>(C::NST);
#pragma unroll
            for (int b = 0; b < P / R; ++b)
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int nn = t + T * b + NS * r;
                    float2 val = cscale(w[b * R + r], inv);
                    const int j = (2 * (2 * nn + h) + shift) & (kSlice - 1);
                    if (wnd) {
                        const float2 wj = vec ? __ldg(reinterpret_cast<const float2*>(wnd + j))
                                              : make_float2(__ldg(wnd + j), __ldg(wnd + j + 1));
                        val.x *= wj.x;
                        val.y *= wj.y;
                    }
                    const long long p = p0 + j;
                    if (vec && p >= lo && p + 1 < hi) {
                        atomicAdd(reinterpret_cast<float2*>(yr + p), val);
                    } else {
                        if (p >= lo && p < hi) atomicAdd(yr + p, val.x);
                        if (p + 1 >= lo && p + 1 < hi) atomicAdd(yr + p + 1, val.y);
                    }
                }
        });
    }
}

}  // namespace

int spectrum_twiddle_count() { return kSpecRowsTotal; }

namespace {
template <class C>
void rows_for(float2* out) {
    const double two_pi = 6.283185307179586476925286766559;
    auto w = [&](long e, long base) {
        const double a = -two_pi * (double)(e % base) / (double)base;
        return make_float2((float)std::cos(a), (float)std::sin(a));
    };
    for (int s = 2; s <= C::NST; ++s) {
        const int R = sR<C>(s), NS = sNS<C>(s), off = sOff<C>(s);
        const long base = (long)NS * R;
        if (sSplit<C>(s)) {
            for (int r = 0; r < R; ++r)
                for (int k = 0; k < 32; ++k) out[off + r * 32 + k] = w((long)r * k, base);
            for (int r = 0; r < R; ++r)
                for (int k = 0; k < NS / 32; ++k)
                    out[off + R * 32 + r * (NS / 32) + k] = w((long)r * 32 * k, base);
        } else {
            for (int r = 1; r < R; ++r)
                for (int k = 0; k < NS; ++k) out[off + (r - 1) * NS + k] = w((long)r * k, base);
        }
    }
}
}  // namespace

// stage twiddle rows of every schedule, forward sign, double precision
// rounded once
void spectrum_twiddle_rows(float2* out) {
    rows_for<S16k32>(out + rowsOff<S16k32>());
    rows_for<S16k16>(out + rowsOff<S16k16>());
    rows_for<S8k32>(out + rowsOff<S8k32>());
    rows_for<S8k16>(out + rowsOff<S8k16>());
}

#ifndef FCQT_SPEC_PREFETCH
#define FCQT_SPEC_PREFETCH 1
#endif

namespace {
// CTAs resident at once on the current device (one spectrum CTA per SM)
int wave_ctas() {
    if (!FCQT_SPEC_PREFETCH) return 0;
    static int sms[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (sms[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return 0;
        sms[dev] = n;
    }
    return sms[dev];
}
}  // namespace

namespace {
// loss = scale * sum of n partial sums: thread i adds partials i, i + 256, ...
// in order, then a fixed halving tree (one CTA, deterministic)
__global__ void __launch_bounds__(256, 1)
sqerr_finish_kernel(const float* __restrict__ partial, int n, float scale, float* loss) {
    pdl_launch_dependents();
    __shared__ float red[256];
    pdl_wait();   // the partials of the previous kernel are complete
    const int t = threadIdx.x;
    float a = 0.f;
    for (int i = t; i < n; i += 256) a += partial[i];
    red[t] = a;
    __syncthreads();
#pragma unroll
    for (int w = 128; w > 0; w >>= 1) {
        if (t < w) red[t] += red[t + w];
        __syncthreads();
    }
    if (t == 0) *loss = scale * red[0];
}
}  // namespace

cudaError_t launch_sqerr_finish(const float* partial, int n, float scale, float* loss,
                                cudaStream_t s) {
    return launch_pdl(n / 2 <= kPdlMaxBatch, sqerr_finish_kernel, dim3(1), dim3(256), 0, s,
                      partial, n, scale, loss);
}

namespace {
template <class G>
cudaError_t spectrum_fwd_geo(const SigMap& in, float2* X, const SpecTables& st, int batch,
                             cudaStream_t s) {
    using C = CFg<G>;
    const int ahead = wave_ctas();
    auto go = [&](auto kern) {
        return launch_pdl(batch <= kPdlMaxBatch, kern, dim3(spectrum_ctas(batch)), dim3(C::T),
                          smemOf<C>(), s, in, X, st.hi, st.lo, st.rows, ahead);
    };
    if (in.S > 0) return go(spectrum_fwd_kernel<kSigSliced, G>);
    if (in.target) return go(spectrum_fwd_kernel<kSigSqErr, G>);
    return go(spectrum_fwd_kernel<kSigPlain, G>);
}

template <class G>
cudaError_t spectrum_inv_geo(const float2* E, const InvTab& tab, const SigMap& out,
                             const SpecTables& st, int batch, cudaStream_t s) {
    using C = CIg<G>;
    const int ahead = wave_ctas();
    auto go = [&](auto kern) {
        return launch_pdl(batch <= kPdlMaxBatch, kern, dim3(spectrum_ctas(batch)), dim3(C::T),
                          smemOf<C>(), s, E, tab.qmask, out, st.hi, st.lo, st.rows,
                          tab.nplanes, ahead);
    };
    if (out.S > 0) return go(spectrum_inv_kernel<kSigSliced, G>);
    if (out.partial) return go(spectrum_inv_kernel<kSigSqErr, G>);
    return go(spectrum_inv_kernel<kSigPlain, G>);
}

template <class G>
cudaError_t spectrum_attributes_geo() {
    const void* fwd[] = {(const void*)spectrum_fwd_kernel<kSigPlain, G>,
                         (const void*)spectrum_fwd_kernel<kSigSliced, G>,
                         (const void*)spectrum_fwd_kernel<kSigSqErr, G>};
    const void* inv[] = {(const void*)spectrum_inv_kernel<kSigPlain, G>,
                         (const void*)spectrum_inv_kernel<kSigSliced, G>,
                         (const void*)spectrum_inv_kernel<kSigSqErr, G>};
    for (const void* f : fwd) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             smemOf<CFg<G>>());
        if (e != cudaSuccess) return e;
    }
    for (const void* f : inv) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             smemOf<CIg<G>>());
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}
}  // namespace

cudaError_t launch_spectrum_fwd(const SigMap& in, float2* X, const SpecTables& st, int batch,
                                cudaStream_t s) {
    if (batch <= 0) return cudaSuccess;
    return st.nslice == 32768 ? spectrum_fwd_geo<Geo<32768>>(in, X, st, batch, s)
                              : spectrum_fwd_geo<Geo<65536>>(in, X, st, batch, s);
}

cudaError_t launch_spectrum_inv(const float2* E, const InvTab& tab, const SigMap& out,
                                const SpecTables& st, int batch, cudaStream_t s) {
    if (batch <= 0) return cudaSuccess;
    return st.nslice == 32768 ? spectrum_inv_geo<Geo<32768>>(E, tab, out, st, batch, s)
                              : spectrum_inv_geo<Geo<65536>>(E, tab, out, st, batch, s);
}

cudaError_t init_spectrum_attributes() {
    cudaError_t e = spectrum_attributes_geo<Geo<65536>>();
    return e == cudaSuccess ? spectrum_attributes_geo<Geo<32768>>() : e;
}

}  // namespace fcqt
