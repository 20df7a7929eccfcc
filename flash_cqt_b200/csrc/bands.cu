// Band engine: the per-band native-length transforms of the constant-Q
// analysis and synthesis (block lengths M = 32 ... 2048, 154 bands a slice).
//
// bands_fwd (analysis engine; also the transpose of the synthesis):
//   gather   v[m] = gain[m] * X~[src[m]]        (window / routing table)
//   DFT      coef[n] = sum_m v[m] e^{+2 pi i m n / M}   (1/M folded in gain)
//   store    natural-order coefficient heap, coalesced
// bands_inv (synthesis engine; also the transpose of the analysis):
//   load     coefficient heap, coalesced
//   DFT      S[m] = sum_n coef[n] e^{-2 pi i m n / M}
//   scatter  E[dest[m]] = (Re S gre[m], Im S gim[m])   one owned slot per tap
//
// Replaces the reference's radix band engine (radix_impl.cuh:146-443), which
// runs warp-shuffle radix-8/16/32 butterflies, one CTA per (band, slice):
// here each thread holds 32 points in registers and runs whole radix-32 /
// radix-2..32 butterflies (no shuffles), the stages exchange through padded
// shared memory, and one 256-thread CTA processes 8192 points = 8192 / M
// (band, slice) instances of one block length, so small bands batch up and
// the tables are reused across the slices of a CTA.
#include "engine.cuh"
#include "internal.h"

namespace fcqt {

namespace {

constexpr int kP = 32;
constexpr int kBandSmem = (kBandCap / 32) * 33 * 8;   // padded(kBandCap) float2

struct Tw2048 {
    const float2* w;
    __device__ __forceinline__ float2 operator()(int e) const { return __ldg(w + (e & 2047)); }
};

template <int M> struct Sched;       // stage radices per block length
template <> struct Sched<32>   { static constexpr int R1 = 32, R2 = 1,  R3 = 1; };
template <> struct Sched<64>   { static constexpr int R1 = 32, R2 = 2,  R3 = 1; };
template <> struct Sched<128>  { static constexpr int R1 = 32, R2 = 4,  R3 = 1; };
template <> struct Sched<256>  { static constexpr int R1 = 32, R2 = 8,  R3 = 1; };
template <> struct Sched<512>  { static constexpr int R1 = 32, R2 = 16, R3 = 1; };
template <> struct Sched<1024> { static constexpr int R1 = 32, R2 = 32, R3 = 1; };
template <> struct Sched<2048> { static constexpr int R1 = 32, R2 = 32, R3 = 2; };

struct Inst {
    int t;        // thread index within the instance
    int il;       // instance index within the CTA
    bool valid;
    int slice;
    int band;
    int off;      // heap offset of the band
};

template <int M>
__device__ __forceinline__ Inst locate(const BandCommon& bc, const BandSched& sc, int c) {
    constexpr int T = M / kP;
    constexpr int IPC = kBandThreads / T;
    Inst in;
    in.t = threadIdx.x % T;
    in.il = threadIdx.x / T;
    const int inst = (blockIdx.x - sc.cta0[c]) * IPC + in.il;
    const int B = sc.batch;
    in.valid = inst < sc.nb[c] * B;
    in.slice = in.valid ? inst % B : 0;
    in.band = in.valid ? __ldg(bc.band_list + sc.first[c] + inst / B) : 0;
    in.off = in.valid ? __ldg(bc.band_off + in.band) : 0;
    return in;
}

// remaining stages (2 and 3) of a block-length-M transform after stage 1's
// DFT; the last stage's outputs (index n = j + r M / R_last) go to `emit`
template <int M, int S, class Emit>
__device__ __forceinline__ void band_rest(float2 (&v)[kP], float2* buf, int t,
                                          const Tw2048& tw, Emit emit) {
    constexpr int T = M / kP;
    constexpr int R1 = Sched<M>::R1, R2 = Sched<M>::R2, R3 = Sched<M>::R3;
    using std::integral_constant;
    if constexpr (R2 == 1) {
        emit(v, integral_constant<int, R1>{}, integral_constant<int, 1>{});
    } else {
        stage_store<M, T, R1, 1>(v, buf, t);
        __syncthreads();
        stage_load<M, T, R2>(v, buf, t);
        __syncthreads();
        stage_compute<M, T, R2, R1, S, 2048>(v, t, tw);
        if constexpr (R3 == 1) {
            emit(v, integral_constant<int, R2>{}, integral_constant<int, R1>{});
        } else {
            stage_store<M, T, R2, R1>(v, buf, t);
            __syncthreads();
            stage_load<M, T, R3>(v, buf, t);
            __syncthreads();
            stage_compute<M, T, R3, R1 * R2, S, 2048>(v, t, tw);
            emit(v, integral_constant<int, R3>{}, integral_constant<int, R1 * R2>{});
        }
    }
}

__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
    const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(sa), "l"(gmem));
}

__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

template <int M>
__device__ void band_fwd(const float2* __restrict__ X, const FwdTab& tab, const BandCommon& bc,
                         const BandSched& sc, int c, CoefPtr out, float2* smem) {
    constexpr int T = M / kP;
    constexpr int R1 = Sched<M>::R1;
    const Inst in = locate<M>(bc, sc, c);
    const int t = in.t;
    float2* buf = smem + in.il * padded(M);
    const Tw2048 tw{bc.tw2048};
    const float2* Xs = X + (long)in.slice * kPlaneStride;

    // stage the band's contiguous spectrum segment (<= M bins) into shared
    // memory with asynchronous copies, independent of the tap-table loads
    int lo = 0;
    if (in.valid) {
        const int2 sg = __ldg(tab.seg + in.band);
        lo = sg.x;
        for (int i = t; i < sg.y; i += T) cp_async8(buf + PADI(i), Xs + lo + i);
    }
    // stage 1 taps: element r of butterfly b is tap t + T b + r M / R1
    int src[kP];
    float gain[kP];
#pragma unroll
    for (int b = 0; b < kP / R1; ++b)
#pragma unroll
        for (int r = 0; r < R1; ++r) {
            const int m = in.off + t + T * b + r * (M / R1);
            src[b * R1 + r] = in.valid ? __ldg(tab.src + m) : -1;
            gain[b * R1 + r] = in.valid ? __ldg(tab.gain + m) : 0.f;
        }
    cp_async_wait_all();
    __syncthreads();
    float2 v[kP];
#pragma unroll
    for (int i = 0; i < kP; ++i) {
        const int s = src[i];
        float2 val = make_float2(0.f, 0.f);
        if (s >= 0) {
            float2 xv = buf[PADI((s & 0xFFFF) - lo)];
            if (s & 0x10000) xv.y = -xv.y;
            val = cscale(xv, gain[i]);
        }
        v[i] = val;
    }
    __syncthreads();   // the segment is dead; stage 1 reuses the buffer
    static_for<0, kP / R1>([&](auto Bb) {
        dft<R1, +1, decltype(Bb)::value * R1, 1>(v);
    });

    const long hb = (long)in.slice * bc.ncoef + in.off;
    band_rest<M, +1>(v, buf, t, tw, [&](float2 (&w)[kP], auto Rc, auto NSc) {
        constexpr int R = decltype(Rc)::value, NS = decltype(NSc)::value;
        if (!in.valid) return;
        // last stage: j = t + T b < NS, output index n = j + r NS
#pragma unroll
        for (int b = 0; b < kP / R; ++b)
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int n = t + T * b + r * NS;
                const float2 val = w[b * R + r];
                if (out.interleaved) {
                    reinterpret_cast<float2*>(out.re)[hb + n] = val;
                } else {
                    out.re[hb + n] = val.x;
                    out.im[hb + n] = val.y;
                }
            }
    });
}

template <int M>
__device__ void band_inv(CoefPtr in_c, const InvTab& tab, const BandCommon& bc,
                         const BandSched& sc, int c, float2* __restrict__ E, float2* smem) {
    constexpr int T = M / kP;
    constexpr int R1 = Sched<M>::R1;
    const Inst in = locate<M>(bc, sc, c);
    const int t = in.t;
    float2* buf = smem + in.il * padded(M);
    const Tw2048 tw{bc.tw2048};
    const long hb = (long)in.slice * bc.ncoef + in.off;

    float2 v[kP];
#pragma unroll
    for (int b = 0; b < kP / R1; ++b)
#pragma unroll
        for (int r = 0; r < R1; ++r) {
            const int n = t + T * b + r * (M / R1);
            float2 val = make_float2(0.f, 0.f);
            if (in.valid) {
                if (in_c.interleaved) {
                    val = __ldg(reinterpret_cast<const float2*>(in_c.re) + hb + n);
                } else {
                    val.x = __ldg(in_c.re + hb + n);
                    val.y = __ldg(in_c.im + hb + n);
                }
            }
            v[b * R1 + r] = val;
        }
    static_for<0, kP / R1>([&](auto Bb) {
        dft<R1, -1, decltype(Bb)::value * R1, 1>(v);
    });

    float2* Es = E + (long)in.slice * tab.nplanes * kPlaneStride;
    band_rest<M, -1>(v, buf, t, tw, [&](float2 (&w)[kP], auto Rc, auto NSc) {
        constexpr int R = decltype(Rc)::value, NS = decltype(NSc)::value;
        if (!in.valid) return;
#pragma unroll
        for (int b = 0; b < kP / R; ++b)
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int m = in.off + t + T * b + r * NS;
                const int d = __ldg(tab.dest + m);
                if (d >= 0) {
                    const float2 val = w[b * R + r];
                    Es[d] = make_float2(val.x * __ldg(tab.gre + m), val.y * __ldg(tab.gim + m));
                }
            }
    });
}

__device__ __forceinline__ int find_class(const BandSched& sc) {
    int c = 0;
    while (c + 1 < sc.ncls && (int)blockIdx.x >= sc.cta0[c + 1]) ++c;
    return c;
}

__global__ void __launch_bounds__(kBandThreads, 2)
bands_fwd_kernel(const float2* __restrict__ X, FwdTab tab, BandCommon bc, BandSched sc,
                 CoefPtr out) {
    extern __shared__ float4 smem_raw[];
    float2* smem = reinterpret_cast<float2*>(smem_raw);
    const int c = find_class(sc);
    switch (sc.M[c]) {
    case 2048: band_fwd<2048>(X, tab, bc, sc, c, out, smem); break;
    case 1024: band_fwd<1024>(X, tab, bc, sc, c, out, smem); break;
    case 512:  band_fwd<512>(X, tab, bc, sc, c, out, smem); break;
    case 256:  band_fwd<256>(X, tab, bc, sc, c, out, smem); break;
    case 128:  band_fwd<128>(X, tab, bc, sc, c, out, smem); break;
    case 64:   band_fwd<64>(X, tab, bc, sc, c, out, smem); break;
    case 32:   band_fwd<32>(X, tab, bc, sc, c, out, smem); break;
    default: break;
    }
}

__global__ void __launch_bounds__(kBandThreads, 2)
bands_inv_kernel(CoefPtr in, InvTab tab, BandCommon bc, BandSched sc, float2* __restrict__ E) {
    extern __shared__ float4 smem_raw[];
    float2* smem = reinterpret_cast<float2*>(smem_raw);
    const int c = find_class(sc);
    switch (sc.M[c]) {
    case 2048: band_inv<2048>(in, tab, bc, sc, c, E, smem); break;
    case 1024: band_inv<1024>(in, tab, bc, sc, c, E, smem); break;
    case 512:  band_inv<512>(in, tab, bc, sc, c, E, smem); break;
    case 256:  band_inv<256>(in, tab, bc, sc, c, E, smem); break;
    case 128:  band_inv<128>(in, tab, bc, sc, c, E, smem); break;
    case 64:   band_inv<64>(in, tab, bc, sc, c, E, smem); break;
    case 32:   band_inv<32>(in, tab, bc, sc, c, E, smem); break;
    default: break;
    }
}

}  // namespace

BandSched make_sched(int ncls, const int* M, const int* nb, const int* first, int batch) {
    BandSched sc{};
    sc.ncls = ncls;
    sc.batch = batch;
    int cta = 0;
    for (int c = 0; c < ncls; ++c) {
        sc.M[c] = M[c];
        sc.nb[c] = nb[c];
        sc.first[c] = first[c];
        sc.cta0[c] = cta;
        const int ipc = kBandCap / M[c];
        const long inst = (long)nb[c] * batch;
        cta += (int)((inst + ipc - 1) / ipc);
    }
    sc.cta0[ncls] = cta;
    return sc;
}

cudaError_t launch_bands_fwd(const float2* X, const FwdTab& tab, const BandCommon& bc,
                             const BandSched& sc, CoefPtr out, cudaStream_t s) {
    const int grid = sc.cta0[sc.ncls];
    if (grid <= 0) return cudaSuccess;
    bands_fwd_kernel<<<grid, kBandThreads, kBandSmem, s>>>(X, tab, bc, sc, out);
    return cudaGetLastError();
}

cudaError_t launch_bands_inv(CoefPtr in, const InvTab& tab, const BandCommon& bc,
                             const BandSched& sc, float2* E, cudaStream_t s) {
    const int grid = sc.cta0[sc.ncls];
    if (grid <= 0) return cudaSuccess;
    bands_inv_kernel<<<grid, kBandThreads, kBandSmem, s>>>(in, tab, bc, sc, E);
    return cudaGetLastError();
}

cudaError_t init_band_attributes() {
    cudaError_t e = cudaFuncSetAttribute(bands_fwd_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kBandSmem);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(bands_inv_kernel,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, kBandSmem);
}

}  // namespace fcqt
