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
// shared memory, runs it as Stockham stages 32 x 32 x 16 (512 threads, 32
// points each), and then untangles the (q, L - q) bin pairs of its parity --
// which are all local -- into the real spectrum X[q] (spectral recovery of
// fused.py:311-328, done once per bin instead of once per router tap).
// The inverse mirrors it: each CTA rebuilds the packed spectrum from the
// colour planes on the fly (quads {n, 16384 - n, 16384 + n, 32768 - n} close
// under both the retangle and the DIF maps), forms its DIF half, runs the
// inverse Stockham stages and stores z[2m + h] de-interleaved into y.
#include "engine.cuh"
#include "internal.h"

namespace fcqt {

namespace {

constexpr int kSpecP = 32;
constexpr int kSpecT = kSpecThreads;
constexpr int kSpecSmem = padded(kQuarter) * 8 + 2 * 256 * 8;

struct Tw64k {
    const float2* hi;
    const float2* lo;
    __device__ __forceinline__ float2 operator()(int e) const { return tw64k(hi, lo, e); }
};

__device__ __forceinline__ void load_twiddles(float2* hi, float2* lo,
                                              const float2* ghi, const float2* glo) {
    const int t = threadIdx.x;
    if (t < 256) hi[t] = ghi[t];
    else if (t < 512) lo[t - 256] = glo[t - 256];
}

// the three Stockham stages of the 16384-point sub-transform after stage 1's
// DFT; S = -1 forward (result left in shared memory, natural order),
// S = +1 inverse (result handed to the caller's store functor)
template <int S, class Store>
__device__ __forceinline__ void quarter_stages_2_3(float2 (&v)[kSpecP], float2* buf,
                                                   const Tw64k& tw, Store store) {
    const int t = threadIdx.x;
    // stage 1 output (R = 32, NS = 1)
    stage_store<kQuarter, kSpecT, 32, 1>(v, buf, t);
    __syncthreads();
    // stage 2: R = 32, NS = 32
    stage_load<kQuarter, kSpecT, 32>(v, buf, t);
    __syncthreads();
    stage_compute<kQuarter, kSpecT, 32, 32, S, 65536>(v, t, tw);
    stage_store<kQuarter, kSpecT, 32, 32>(v, buf, t);
    __syncthreads();
    // stage 3: R = 16, NS = 1024, two butterflies per thread
    stage_load<kQuarter, kSpecT, 16>(v, buf, t);
    __syncthreads();
    stage_compute<kQuarter, kSpecT, 16, 1024, S, 65536>(v, t, tw);
    store(v);
}

__global__ void __launch_bounds__(kSpecThreads, 1)
spectrum_fwd_kernel(const float* __restrict__ x, float2* __restrict__ X,
                    const float2* __restrict__ ghi, const float2* __restrict__ glo) {
    extern __shared__ float4 smem_raw[];
    float2* buf = reinterpret_cast<float2*>(smem_raw);
    float2* hi = buf + padded(kQuarter);
    float2* lo = hi + 256;
    const int h = blockIdx.x & 1;
    const long slice = blockIdx.x >> 1;
    const int t = threadIdx.x;
    load_twiddles(hi, lo, ghi, glo);
    __syncthreads();
    const Tw64k tw{hi, lo};

    // stage 1 inputs straight from global: the radix-2 DIF split of z
    const float2* z = reinterpret_cast<const float2*>(x + slice * kSlice);
    float2 v[kSpecP];
#pragma unroll
    for (int r = 0; r < 32; ++r) {
        const int n = t + kSpecT * r;
        const float2 a = __ldg(z + n);
        const float2 b = __ldg(z + n + kQuarter);
        v[r] = h == 0 ? cadd(a, b) : cmul(csub(a, b), tw(2 * n));
    }
    dft<32, -1, 0, 1>(v);
    quarter_stages_2_3<-1>(v, buf, tw, [&](float2 (&w)[kSpecP]) {
        stage_store<kQuarter, kSpecT, 16, 1024>(w, buf, t);
    });
    __syncthreads();

    // untangle the (q, L - q) pairs of this parity: X[q] = E + W_N^q O
    float2* Xs = X + slice * kPlaneStride;
    const int npairs = h == 0 ? kQuarter / 2 + 1 : kQuarter / 2;
    for (int kp = t; kp < npairs; kp += kSpecT) {
        const int kq = h == 0 ? ((kQuarter - kp) & (kQuarter - 1)) : (kQuarter - 1 - kp);
        const float2 zq = buf[PADI(kp)];
        const float2 zb = buf[PADI(kq)];
        const int q = 2 * kp + h;
        const float2 w = tw(q);
        const float2 sq = cadd(zq, cconj(zb));   // 2 E[q]
        const float2 dq = csub(zq, cconj(zb));   // 2 i O[q] / ... (before W)
        const float2 wd = cmul(w, dq);
        // X[q] = (sq - i w dq) / 2
        Xs[q] = make_float2(0.5f * (sq.x + wd.y), 0.5f * (sq.y - wd.x));
        if (kq != kp || q == 0) {
            // X[L - q] = (conj(sq) + i conj(w) conj(dq) ... ) / 2, written via
            // the partner's own sums: sb = zb + conj zq, db = zb - conj zq
            const float2 sb = cconj(sq);
            const float2 db = make_float2(-dq.x, dq.y);
            const float2 wdb = cmulc(db, w);     // conj(w) * db
            Xs[kHalf - q] = make_float2(0.5f * (sb.x - wdb.y), 0.5f * (sb.y + wdb.x));
        }
    }
}

// F[q] from the colour planes, planes flagged in mask[q], fixed plane order.
// Planes 0 and 1 cover almost every bin, so they are loaded unconditionally
// (in parallel with the mask) and selected; planes 2 and 3 are rare.
__device__ __forceinline__ float2 plane_sum(const float2* __restrict__ Es,
                                            const unsigned char* __restrict__ mask,
                                            int q, int nplanes) {
    const unsigned mk = __ldg(mask + q);
    const float2 e0 = Es[q];
    const float2 e1 = nplanes > 1 ? Es[kPlaneStride + q] : make_float2(0.f, 0.f);
    float2 acc = make_float2(0.f, 0.f);
    if (mk & 1u) acc = cadd(acc, e0);
    if (mk & 2u) acc = cadd(acc, e1);
    if (mk & 4u) acc = cadd(acc, Es[2 * kPlaneStride + q]);
    if (mk & 8u) acc = cadd(acc, Es[3 * kPlaneStride + q]);
    return acc;
}

// packed spectrum Zs[q] = E + i O, E = (a + conj b)/2, O = (a - conj b) W_N^-q / 2
__device__ __forceinline__ float2 retangle(float2 a, float2 b, float2 wq) {
    const float2 e = make_float2(0.5f * (a.x + b.x), 0.5f * (a.y - b.y));
    const float2 d = make_float2(0.5f * (a.x - b.x), 0.5f * (a.y + b.y));
    const float2 o = cmulc(d, wq);               // d * conj(W_N^q)
    return make_float2(e.x - o.y, e.y + o.x);
}

__global__ void __launch_bounds__(kSpecThreads, 1)
spectrum_inv_kernel(const float2* __restrict__ E, const unsigned char* __restrict__ mask,
                    float* __restrict__ y, const float2* __restrict__ ghi,
                    const float2* __restrict__ glo, int nplanes) {
    extern __shared__ float4 smem_raw[];
    float2* buf = reinterpret_cast<float2*>(smem_raw);
    float2* hi = buf + padded(kQuarter);
    float2* lo = hi + 256;
    const int h = blockIdx.x & 1;
    const long slice = blockIdx.x >> 1;
    const int t = threadIdx.x;
    load_twiddles(hi, lo, ghi, glo);
    __syncthreads();
    const Tw64k tw{hi, lo};
    const float2* Es = E + slice * (long)(nplanes * kPlaneStride);

    // quads {n, L - n, Q + n, Q - n}: four bins in, u_h[n] and u_h[Q - n] out
    for (int n = t; n <= kQuarter / 2; n += kSpecT) {
        const int m = (kQuarter - n) & (kQuarter - 1);
        float2 fA = plane_sum(Es, mask, n, nplanes);
        float2 fB = plane_sum(Es, mask, kHalf - n, nplanes);
        const float2 fC = plane_sum(Es, mask, kQuarter + n, nplanes);
        const float2 fD = plane_sum(Es, mask, kQuarter - n, nplanes);
        if (n == 0) {  // irfft ignores the imaginary parts of DC and Nyquist
            fA.y = 0.f;
            fB.y = 0.f;
        }
        const float2 z0 = retangle(fA, fB, tw(n));
        const float2 z1 = retangle(fC, fD, tw(kQuarter + n));
        float2 un = h == 0 ? cadd(z0, z1) : cmulc(csub(z0, z1), tw(2 * n));
        buf[PADI(n)] = un;
        if (m != n) {
            const float2 z2 = retangle(fD, fC, tw(m));
            const float2 z3 = retangle(fB, fA, tw(kQuarter + m));
            buf[PADI(m)] = h == 0 ? cadd(z2, z3) : cmulc(csub(z2, z3), tw(2 * m));
        }
    }
    __syncthreads();

    float2 v[kSpecP];
    stage_load<kQuarter, kSpecT, 32>(v, buf, t);
    __syncthreads();
    dft<32, +1, 0, 1>(v);
    float2* ys = reinterpret_cast<float2*>(y + slice * kSlice);
    const float inv = 1.0f / (float)kHalf;
    quarter_stages_2_3<+1>(v, buf, tw, [&](float2 (&w)[kSpecP]) {
        // last stage output index n = j + 1024 r (NS = 1024 = M / R)
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                const int nn = t + kSpecT * b + 1024 * r;
                ys[2 * nn + h] = cscale(w[b * 16 + r], inv);
            }
    });
}

}  // namespace

cudaError_t launch_spectrum_fwd(const float* x, float2* X, const float2* tw_hi,
                                const float2* tw_lo, int batch, cudaStream_t s) {
    if (batch <= 0) return cudaSuccess;
    spectrum_fwd_kernel<<<2 * batch, kSpecThreads, kSpecSmem, s>>>(x, X, tw_hi, tw_lo);
    return cudaGetLastError();
}

cudaError_t launch_spectrum_inv(const float2* E, const InvTab& tab, float* y,
                                const float2* tw_hi, const float2* tw_lo,
                                int batch, cudaStream_t s) {
    if (batch <= 0) return cudaSuccess;
    spectrum_inv_kernel<<<2 * batch, kSpecThreads, kSpecSmem, s>>>(
        E, tab.mask, y, tw_hi, tw_lo, tab.nplanes);
    return cudaGetLastError();
}

cudaError_t init_spectrum_attributes() {
    cudaError_t e = cudaFuncSetAttribute(spectrum_fwd_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSpecSmem);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(spectrum_inv_kernel,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, kSpecSmem);
}

}  // namespace fcqt
