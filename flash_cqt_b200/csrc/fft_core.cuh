// Register-level DFT building blocks for the sm_100a FFT engines.
//
// Everything here works on float2 complex values held in registers.  A DFT of
// radix R (2, 4, 8, 16, 32, 64) is written as a composite R = R1 x R2
// ("four-step" inside one thread): R2 DFTs of length R1 over the strided
// inputs, an internal twiddle W_R^(n2 k1), then R1 DFTs of length R2.  The
// internal twiddles are compile-time constants (cos(2 pi j / 64) evaluated in
// double precision when this header was generated and rounded to float once),
// so after unrolling every multiply by 1, -i or (1 - i)/sqrt(2) folds away.
//
// Sign convention: S = -1 is the forward transform sum x[n] e^{-2 pi i nk/R},
// S = +1 the unnormalised inverse.
#pragma once
#include <cuda_runtime.h>
#include <type_traits>

namespace fcqt {

// cos(2 pi j / 64), j = 0..63
constexpr double kCos64[64] = {
    1,
    0.99518472667219693,
    0.98078528040323043,
    0.95694033573220882,
    0.92387953251128674,
    0.88192126434835505,
    0.83146961230254524,
    0.77301045336273699,
    0.70710678118654757,
    0.63439328416364549,
    0.55557023301960229,
    0.47139673682599781,
    0.38268343236508984,
    0.29028467725446233,
    0.19509032201612833,
    0.09801714032956077,
    6.123233995736766e-17,
    -0.098017140329560645,
    -0.19509032201612819,
    -0.29028467725446216,
    -0.38268343236508973,
    -0.4713967368259977,
    -0.55557023301960196,
    -0.63439328416364538,
    -0.70710678118654746,
    -0.77301045336273699,
    -0.83146961230254535,
    -0.88192126434835494,
    -0.92387953251128674,
    -0.95694033573220882,
    -0.98078528040323043,
    -0.99518472667219682,
    -1,
    -0.99518472667219693,
    -0.98078528040323043,
    -0.95694033573220894,
    -0.92387953251128685,
    -0.88192126434835505,
    -0.83146961230254546,
    -0.7730104533627371,
    -0.70710678118654768,
    -0.63439328416364593,
    -0.55557023301960218,
    -0.47139673682599786,
    -0.38268343236509034,
    -0.29028467725446244,
    -0.19509032201612866,
    -0.098017140329560451,
    -1.8369701987210297e-16,
    0.09801714032956009,
    0.1950903220161283,
    0.29028467725446205,
    0.38268343236509,
    0.47139673682599759,
    0.55557023301960184,
    0.6343932841636456,
    0.70710678118654735,
    0.77301045336273666,
    0.83146961230254524,
    0.88192126434835483,
    0.92387953251128652,
    0.95694033573220882,
    0.98078528040323032,
    0.99518472667219693
};

template <int I, int N, class F>
__device__ __forceinline__ void static_for(F&& f) {
    if constexpr (I < N) {
        f(std::integral_constant<int, I>{});
        static_for<I + 1, N>(f);
    }
}

// Complex add and subtract as sm_100 packed two-lane fp32 instructions (one
// instruction for both components; each lane rounds as the scalar operation,
// and a - b is formed exactly as b * -1 + a).  The complex product is
// a.x (b.x, b.y) + a.y (-b.y, b.x) as one packed multiply and one packed
// fused multiply-add (one rounding after the multiply, one after the add, as
// the scalar form, with the roles of the two products swapped).
// FCQT_F32X2=0 builds the scalar forms.
#ifndef FCQT_F32X2
#define FCQT_F32X2 1
#endif
#if FCQT_F32X2
__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) {
    return __ffma2_rn(b, make_float2(-1.f, -1.f), a);
}
#else
__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
#endif
__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
#if FCQT_F32X2
    const float2 t = __fmul2_rn(make_float2(a.x, a.x), b);
    return __ffma2_rn(make_float2(a.y, a.y), make_float2(-b.y, b.x), t);
#else
    return make_float2(fmaf(a.x, b.x, -a.y * b.y), fmaf(a.x, b.y, a.y * b.x));
#endif
}
// a * conj(b)
__device__ __forceinline__ float2 cmulc(float2 a, float2 b) {
    return make_float2(fmaf(a.x, b.x, a.y * b.y), fmaf(a.y, b.x, -a.x * b.y));
}
__device__ __forceinline__ float2 cconj(float2 a) { return make_float2(a.x, -a.y); }
__device__ __forceinline__ float2 cscale(float2 a, float s) { return make_float2(a.x * s, a.y * s); }

// a * (S i): S = -1 -> multiply by -i, S = +1 -> by +i
template <int S>
__device__ __forceinline__ float2 mul_si(float2 a) {
    if constexpr (S < 0) return make_float2(a.y, -a.x);
    else return make_float2(-a.y, a.x);
}

// y1 = t + S i d and y3 = t - S i d, per component (the swap and the signs
// fold into scalar adds)
template <int S>
__device__ __forceinline__ void rot_pair(float2 t, float2 d, float2& y1, float2& y3) {
    if constexpr (S < 0) {
        y1 = make_float2(t.x + d.y, t.y - d.x);
        y3 = make_float2(t.x - d.y, t.y + d.x);
    } else {
        y1 = make_float2(t.x - d.y, t.y + d.x);
        y3 = make_float2(t.x + d.y, t.y - d.x);
    }
}

// multiply by the compile-time twiddle W_R^E = exp(S 2 pi i E / R)
template <int R, int E, int S>
__device__ __forceinline__ float2 twc(float2 a) {
    constexpr int e = ((E % R) + R) % R;
    if constexpr (e == 0) {
        return a;
    } else if constexpr ((4 * e) % R == 0) {
        constexpr int q = 4 * e / R;  // quarter turns
        if constexpr (q == 1) return mul_si<S>(a);
        else if constexpr (q == 2) return make_float2(-a.x, -a.y);
        else return mul_si<-S>(a);
    } else if constexpr ((8 * e) % R == 0) {
        constexpr int o = 8 * e / R;  // odd octant 1, 3, 5, 7
        constexpr float h = 0.70710678118654752f;
        // (c + S i s) with c = cos(o pi/4), s = sin(o pi/4), |c| = |s| = h
        constexpr float c = (o == 1 || o == 7) ? h : -h;
        constexpr float s = (o == 1 || o == 3) ? h : -h;
        constexpr float ss = S < 0 ? -s : s;
        return make_float2(c * a.x - ss * a.y, c * a.y + ss * a.x);
    } else {
        static_assert(64 % R == 0, "twc: R must divide 64");
        constexpr int j = e * (64 / R);
        constexpr float c = (float)kCos64[j];
        constexpr float s0 = (float)kCos64[(j + 48) % 64];  // sin(2 pi j/64)
        constexpr float s = S < 0 ? -s0 : s0;
        return make_float2(fmaf(c, a.x, -s * a.y), fmaf(c, a.y, s * a.x));
    }
}

// in-register DFT of length R on v[B0 + STRIDE * n], n = 0..R-1, result in
// natural order in the same slots
template <int R, int S, int B0 = 0, int STRIDE = 1, int P>
__device__ __forceinline__ void dft(float2 (&v)[P]);

template <int R>
struct Split {  // R = R1 * R2
    static constexpr int R1 = R == 8 ? 2 : R == 16 ? 4 : R == 32 ? 4 : R == 64 ? 8 : 0;
    static constexpr int R2 = R / (R1 ? R1 : 1);
};

template <int R, int S, int B0, int STRIDE, int P>
__device__ __forceinline__ void dft(float2 (&v)[P]) {
    if constexpr (R == 1) {
        return;
    } else if constexpr (R == 2) {
        float2 a = v[B0], b = v[B0 + STRIDE];
        v[B0] = cadd(a, b);
        v[B0 + STRIDE] = csub(a, b);
    } else if constexpr (R == 4) {
        float2 x0 = v[B0], x1 = v[B0 + STRIDE], x2 = v[B0 + 2 * STRIDE], x3 = v[B0 + 3 * STRIDE];
        float2 t0 = cadd(x0, x2), t1 = csub(x0, x2);
        float2 t2 = cadd(x1, x3), d = csub(x1, x3);
        v[B0] = cadd(t0, t2);
        v[B0 + 2 * STRIDE] = csub(t0, t2);
        rot_pair<S>(t1, d, v[B0 + STRIDE], v[B0 + 3 * STRIDE]);
    } else {
        // R = R1 * R2, input n = R2 n1 + n2, output k = k1 + R1 k2
        constexpr int R1 = Split<R>::R1, R2 = Split<R>::R2;
        static_assert(R1 * R2 == R && R1 > 1, "unsupported radix");
        // step 1: for each n2 a length-R1 DFT over n1 (stride R2 * STRIDE)
        static_for<0, R2>([&](auto N2) {
            constexpr int n2 = decltype(N2)::value;
            dft<R1, S, B0 + n2 * STRIDE, R2 * STRIDE>(v);
        });
        // now slot B0 + (R2 k1 + n2) * STRIDE holds y[n2][k1]; twiddle it
        static_for<1, R2>([&](auto N2) {
            constexpr int n2 = decltype(N2)::value;
            static_for<1, R1>([&](auto K1) {
                constexpr int k1 = decltype(K1)::value;
                constexpr int slot = B0 + (R2 * k1 + n2) * STRIDE;
                v[slot] = twc<R, n2 * k1, S>(v[slot]);
            });
        });
        // step 2: for each k1 a length-R2 DFT over n2 (contiguous run)
        static_for<0, R1>([&](auto K1) {
            constexpr int k1 = decltype(K1)::value;
            dft<R2, S, B0 + R2 * k1 * STRIDE, STRIDE>(v);
        });
        // slot B0 + (R2 k1 + k2) * STRIDE holds X[k1 + R1 k2]: transpose
        float2 t[R];
        static_for<0, R1>([&](auto K1) {
            constexpr int k1 = decltype(K1)::value;
            static_for<0, R2>([&](auto K2) {
                constexpr int k2 = decltype(K2)::value;
                t[k1 + R1 * k2] = v[B0 + (R2 * k1 + k2) * STRIDE];
            });
        });
        static_for<0, R>([&](auto K) {
            constexpr int k = decltype(K)::value;
            v[B0 + k * STRIDE] = t[k];
        });
    }
}

}  // namespace fcqt

namespace fcqt {

// ------------------------------------------------------------------
// DFT with inputs known to be zero (bit n of Z: input n is 0).  The additions
// with a known zero are dropped; results equal dft<R, S, ...> except that a
// zero may come out with the other sign.

template <bool ZA, bool ZB>
__device__ __forceinline__ float2 zadd(float2 a, float2 b) {
    if constexpr (ZA && ZB) return make_float2(0.f, 0.f);
    else if constexpr (ZA) return b;
    else if constexpr (ZB) return a;
    else return cadd(a, b);
}
template <bool ZA, bool ZB>
__device__ __forceinline__ float2 zsub(float2 a, float2 b) {
    if constexpr (ZA && ZB) return make_float2(0.f, 0.f);
    else if constexpr (ZA) return make_float2(-b.x, -b.y);
    else if constexpr (ZB) return a;
    else return csub(a, b);
}

// the bits of Z at inputs B0 + n * STRIDE' that form sub-DFT `n2` of a split
template <int R, unsigned Z, int R2, int n2>
constexpr unsigned sub_mask() {
    unsigned m = 0;
    for (int n1 = 0; n1 < R / R2; ++n1)
        if ((Z >> (R2 * n1 + n2)) & 1u) m |= 1u << n1;
    return m;
}

template <int R, int S, unsigned Z, int B0 = 0, int STRIDE = 1, int P>
__device__ __forceinline__ void dftz(float2 (&v)[P]) {
    constexpr unsigned ALL = (R >= 32) ? 0xFFFFFFFFu : ((1u << R) - 1u);
    if constexpr ((Z & ALL) == 0) {
        dft<R, S, B0, STRIDE>(v);
    } else if constexpr ((Z & ALL) == ALL) {
#pragma unroll
        for (int n = 0; n < R; ++n) v[B0 + n * STRIDE] = make_float2(0.f, 0.f);
    } else if constexpr (R == 2) {
        const float2 a = v[B0], b = v[B0 + STRIDE];
        v[B0] = zadd<(Z & 1u) != 0, (Z & 2u) != 0>(a, b);
        v[B0 + STRIDE] = zsub<(Z & 1u) != 0, (Z & 2u) != 0>(a, b);
    } else if constexpr (R == 4) {
        constexpr bool z0 = Z & 1u, z1 = Z & 2u, z2 = Z & 4u, z3 = Z & 8u;
        const float2 x0 = v[B0], x1 = v[B0 + STRIDE], x2 = v[B0 + 2 * STRIDE],
                     x3 = v[B0 + 3 * STRIDE];
        const float2 t0 = zadd<z0, z2>(x0, x2), t1 = zsub<z0, z2>(x0, x2);
        const float2 t2 = zadd<z1, z3>(x1, x3), d = zsub<z1, z3>(x1, x3);
        constexpr bool zt0 = z0 && z2, zt2 = z1 && z3;
        v[B0] = zadd<zt0, zt2>(t0, t2);
        v[B0 + 2 * STRIDE] = zsub<zt0, zt2>(t0, t2);
        if constexpr (!zt0 && !zt2) {
            rot_pair<S>(t1, d, v[B0 + STRIDE], v[B0 + 3 * STRIDE]);
        } else {
            const float2 t3 = mul_si<S>(d);
            v[B0 + STRIDE] = zadd<zt0, zt2>(t1, t3);
            v[B0 + 3 * STRIDE] = zsub<zt0, zt2>(t1, t3);
        }
    } else {
        constexpr int R1 = Split<R>::R1, R2 = Split<R>::R2;
        static_assert(R1 * R2 == R && R1 > 1, "unsupported radix");
        // step 1: length-R1 DFTs over n1 for each n2, with their zero inputs
        static_for<0, R2>([&](auto N2) {
            constexpr int n2 = decltype(N2)::value;
            dftz<R1, S, sub_mask<R, Z, R2, n2>(), B0 + n2 * STRIDE, R2 * STRIDE>(v);
        });
        // a sub-DFT whose inputs were all zero gives zeros: no twiddle
        static_for<1, R2>([&](auto N2) {
            constexpr int n2 = decltype(N2)::value;
            constexpr bool dead = sub_mask<R, Z, R2, n2>() == ((1u << R1) - 1u);
            if constexpr (!dead) {
                static_for<1, R1>([&](auto K1) {
                    constexpr int k1 = decltype(K1)::value;
                    constexpr int slot = B0 + (R2 * k1 + n2) * STRIDE;
                    v[slot] = twc<R, n2 * k1, S>(v[slot]);
                });
            }
        });
        // step 2: length-R2 DFTs over n2, zero where a whole sub-DFT was
        constexpr unsigned Z2 = [] {
            unsigned m = 0;
            for (int n2 = 0; n2 < R2; ++n2) {
                unsigned s = 0;
                for (int n1 = 0; n1 < R1; ++n1)
                    if ((Z >> (R2 * n1 + n2)) & 1u) s |= 1u << n1;
                if (s == ((1u << R1) - 1u)) m |= 1u << n2;
            }
            return m;
        }();
        static_for<0, R1>([&](auto K1) {
            constexpr int k1 = decltype(K1)::value;
            dftz<R2, S, Z2, B0 + R2 * k1 * STRIDE, STRIDE>(v);
        });
        float2 t[R];
        static_for<0, R1>([&](auto K1) {
            constexpr int k1 = decltype(K1)::value;
            static_for<0, R2>([&](auto K2) {
                constexpr int k2 = decltype(K2)::value;
                t[k1 + R1 * k2] = v[B0 + (R2 * k1 + k2) * STRIDE];
            });
        });
        static_for<0, R>([&](auto K) {
            constexpr int k = decltype(K)::value;
            v[B0 + k * STRIDE] = t[k];
        });
    }
}

}  // namespace fcqt
