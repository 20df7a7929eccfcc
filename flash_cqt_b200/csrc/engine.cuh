// Stockham FFT engine pieces shared by the packed-spectrum and band kernels.
//
// A length-M transform runs as a list of radix-R stages.  Butterfly j of a
// stage with span NS (product of the radices already done) reads
//     in[j + r * M / R]                                       (r = 0..R-1),
// multiplies element r by W_{NS R}^{r k} (k = j mod NS), runs an in-register
// DFT of length R and writes element r to
//     out[(j / NS) * NS * R + k + r * NS].
// After the last stage the result is in natural order, so the first stage can
// read straight from global memory and the last stage can write straight to
// global memory, both coalesced across consecutive j.  Between stages the
// data goes through shared memory with one float2 of padding every 2^SH
// elements (PADI<SH>); with SH = log2(points per thread) every stage's read
// and write pattern is free of bank conflicts (64-bit accesses are served
// per half warp, so the stride-R stores of a radix-R first stage need R
// distinct bank pairs within 16 lanes).
#pragma once
#include "fft_core.cuh"

namespace fcqt {

constexpr int kSlice = 65536;            // samples per slice
constexpr int kHalf = kSlice / 2;        // packed complex length L
constexpr int kQuarter = kHalf / 2;      // per-CTA sub-transform length
constexpr int kPlaneStride = kHalf + 8;  // complex elements per spectrum row / colour plane
constexpr int kMaxPlanes = 4;

template <int SH = 5>
__host__ __device__ constexpr int padded(int n) { return n + (n >> SH); }
template <int SH = 5>
__device__ __forceinline__ int PADI(int i) { return i + (i >> SH); }

// W_65536^e from two 256-entry tables in shared memory: hi[e >> 8] * lo[e & 255]
__device__ __forceinline__ float2 tw64k(const float2* hi, const float2* lo, int e) {
    return cmul(hi[e >> 8], lo[e & 255]);
}

// ---------------------------------------------------------------- stages
// PADI<SH>(a + c) == PADI<SH>(a) + c + (c >> SH) whenever c is a multiple of
// 2^SH, so every shared-memory address below is one per-thread base plus
// compile-time offsets when the stage geometry allows it (it does for all
// but the smallest block lengths); otherwise the generic formula is used.

// Read the inputs of a radix-R stage of length M for butterflies
// j = t + T * b (b < P / R) from a padded shared buffer.
template <int M, int T, int R, int SH, int P>
__device__ __forceinline__ void stage_load(float2 (&v)[P], const float2* buf, int t) {
    constexpr int Q = 1 << SH;
    if constexpr ((T % Q) == 0 && ((M / R) % Q) == 0) {
        const float2* p = buf + PADI<SH>(t);
#pragma unroll
        for (int b = 0; b < P / R; ++b)
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int c = T * b + r * (M / R);
                v[b * R + r] = p[c + (c >> SH)];
            }
    } else {
#pragma unroll
        for (int b = 0; b < P / R; ++b)
#pragma unroll
            for (int r = 0; r < R; ++r)
                v[b * R + r] = buf[PADI<SH>(t + T * b + r * (M / R))];
    }
}

// Write the outputs of a radix-R stage with span NS to a padded shared buffer.
template <int M, int T, int R, int NS, int SH, int P>
__device__ __forceinline__ void stage_store(const float2 (&v)[P], float2* buf, int t) {
    constexpr int Q = 1 << SH;
    // butterfly b of the thread starts at base(t) + T R b when NS divides T
    constexpr bool lin_b = (T % NS) == 0 && ((T * R) % Q) == 0;
    if constexpr (lin_b && (NS % Q) == 0) {
        float2* p = buf + PADI<SH>((t / NS) * NS * R + (t % NS));
#pragma unroll
        for (int b = 0; b < P / R; ++b)
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int c = T * R * b + r * NS;
                p[c + (c >> SH)] = v[b * R + r];
            }
    } else if constexpr (lin_b && NS == 1 && (R % Q) == 0) {
        // base = t R is a multiple of 2^SH and r < R <= ... stays inside one
        // padding period per 2^SH outputs
        float2* p = buf + PADI<SH>(t * R);
#pragma unroll
        for (int b = 0; b < P / R; ++b)
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int c = T * R * b + r;
                p[c + (c >> SH)] = v[b * R + r];
            }
    } else {
#pragma unroll
        for (int b = 0; b < P / R; ++b) {
            const int j = t + T * b;
            const int base = (j / NS) * NS * R + (j % NS);
#pragma unroll
            for (int r = 0; r < R; ++r) buf[PADI<SH>(base + r * NS)] = v[b * R + r];
        }
    }
}

// Twiddle (span NS > 1) and DFT for all butterflies of a thread.  TW(e)
// returns W_{TWBASE}^e in the forward sign; S = +1 conjugates it.
template <int M, int T, int R, int NS, int S, int TWBASE, int P, class TW>
__device__ __forceinline__ void stage_compute(float2 (&v)[P], int t, const TW& tw) {
    static_for<0, P / R>([&](auto Bb) {
        constexpr int b = decltype(Bb)::value;
        if constexpr (NS > 1) {
            const int k = (t + T * b) % NS;
            constexpr int scale = TWBASE / (NS * R);
            static_assert(scale * NS * R == TWBASE, "twiddle base too small");
#pragma unroll
            for (int r = 1; r < R; ++r) {
                float2 w = tw(r * k * scale);
                if constexpr (S > 0) w.y = -w.y;
                v[b * R + r] = cmul(v[b * R + r], w);
            }
        }
        dft<R, S, b * R, 1>(v);
    });
}

}  // namespace fcqt
