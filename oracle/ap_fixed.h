// ap_fixed.h -- a self-contained fixed-point type used ONLY to compile the
// reference Cormorant kernels (kernels/*/kernel/*.cpp) and their C-simulation
// tests with g++ on the CPU, as the parity checker for the CUDA library.
//
// This is test infrastructure, not product code.  The vendor HLS headers the
// reference expects (Vitis HLS 2025.2 `ap_fixed.h`, kernels/matmul/CMakeLists.txt:14-21)
// are not available here, so this file restates the documented arithmetic of
// `ap_fixed<W,I,Q,O,N>` from first principles:
//
//   * value = raw * 2^-(W-I); raw is a W-bit two's-complement integer.
//   * Binary + - * / produce a full-precision result type (no rounding, no
//     overflow):  add/sub -> I = max(I1,I2)+1, F = max(F1,F2);
//                 mul     -> W = W1+W2, I = I1+I2;
//                 div     -> F = F1, raw = (a.raw << F2) / b.raw truncated
//                            toward zero (C integer division), as the
//                            reference scheduler's own model states
//                            (inference-scheduler/src/dtype.py:110-124).
//   * Narrowing into a destination type first quantises the dropped
//     fractional bits with mode Q (AP_TRN = floor toward -inf, the default),
//     then handles integer overflow with mode O (AP_WRAP = keep the low W
//     bits, the default; AP_SAT = clamp to [min, max]).
//   * Compound assignment (+= etc.) forms the exact result, then narrows into
//     the left-hand type.  For ap_fixed<32,16> accumulators this is addition
//     mod 2^32, which the reference relies on (kernels/matmul/include/Config.h.in:20-24).
//   * Conversion to float/double rounds the exact value to nearest-even.
//   * Conversion from float/double is exact before quantisation; NaN converts
//     to 0 and +-Inf is treated as an overflow (AP_SAT clamps, AP_WRAP -> 0).
//     The NaN/Inf rules are this shim's choice: no reference test pins them.
//
// Only what the four reference kernels and their tests use is provided.
#pragma once

#include <cmath>
#include <cstdint>
#include <type_traits>

enum ap_q_mode { AP_RND, AP_RND_ZERO, AP_RND_MIN_INF, AP_RND_INF, AP_RND_CONV, AP_TRN, AP_TRN_ZERO };
enum ap_o_mode { AP_SAT, AP_SAT_ZERO, AP_SAT_SYM, AP_WRAP, AP_WRAP_SM };

namespace apfx {

typedef __int128 wide_t;

template <int W>
struct storage {
    typedef typename std::conditional<(W <= 8), int8_t,
            typename std::conditional<(W <= 16), int16_t,
            typename std::conditional<(W <= 32), int32_t, int64_t>::type>::type>::type type;
};

constexpr int imax(int a, int b) { return a > b ? a : b; }

// floor(v / 2^s) etc. for s >= 1, according to quantisation mode Q.
template <ap_q_mode Q>
inline wide_t shift_quantise(wide_t v, int s) {
    if (s <= 0) return v << (-s);
    if (s > 100) {            // |v| < 2^100 here, so only the sign matters
        v = (v > 0) ? 1 : (v < 0 ? -1 : 0);
        s = 100;
    }
    const wide_t one = 1;
    const wide_t fl = v >> s;                        // floor (arithmetic shift)
    const wide_t rem = v - (fl << s);                // 0 <= rem < 2^s
    const wide_t half = one << (s - 1);
    const bool neg = v < 0;
    switch (Q) {
        case AP_TRN:         return fl;
        case AP_TRN_ZERO:    return (neg && rem != 0) ? fl + 1 : fl;
        case AP_RND:         return (rem >= half) ? fl + 1 : fl;               // half -> +inf
        case AP_RND_MIN_INF: return (rem > half) ? fl + 1 : fl;                // half -> -inf
        case AP_RND_ZERO:    return (rem > half || (rem == half && neg)) ? fl + 1 : fl;
        case AP_RND_INF:     return (rem > half || (rem == half && !neg)) ? fl + 1 : fl;
        case AP_RND_CONV:    return (rem > half || (rem == half && (fl & 1))) ? fl + 1 : fl;
    }
    return fl;
}

// Bring an exact integer v (in destination raw units) into W bits with mode O.
template <int W, ap_o_mode O>
inline int64_t overflow(wide_t v) {
    static_assert(O != AP_WRAP_SM, "AP_WRAP_SM is not provided by this shim");
    const wide_t one = 1;
    const wide_t hi = (one << (W - 1)) - 1;
    const wide_t lo = -(one << (W - 1));
    if (v >= lo && v <= hi) return (int64_t)v;
    switch (O) {
        case AP_SAT:      return (int64_t)(v > hi ? hi : lo);
        case AP_SAT_ZERO: return 0;
        case AP_SAT_SYM:  return (int64_t)(v > hi ? hi : -hi);
        default: {        // AP_WRAP: keep the low W bits, sign-extended
            const uint64_t u = (uint64_t)v;
            if (W == 64) return (int64_t)u;
            const int sh = 64 - W;
            return (int64_t)(u << sh) >> sh;
        }
    }
}

}  // namespace apfx

template <int _AP_W, int _AP_I, ap_q_mode _AP_Q = AP_TRN, ap_o_mode _AP_O = AP_WRAP, int _AP_N = 0>
struct ap_fixed {
    static_assert(_AP_W >= 1 && _AP_W <= 64, "this shim supports widths 1..64");
    static constexpr int W = _AP_W;
    static constexpr int I = _AP_I;
    static constexpr int F = _AP_W - _AP_I;
    typedef typename apfx::storage<_AP_W>::type raw_t;

    raw_t V;

    // Narrow an exact value raw * 2^-fsrc into this type.
    static raw_t narrow(apfx::wide_t raw, int fsrc) {
        const int s = fsrc - F;                     // bits to drop (may be negative)
        apfx::wide_t q;
        if (s > 0) {
            q = apfx::shift_quantise<_AP_Q>(raw, s);
        } else if (s < 0) {
            const int l = -s;
            if (raw == 0) {
                q = 0;
            } else if (_AP_O == AP_WRAP) {
                // only the low W (<= 64) bits survive, so 64-bit arithmetic is exact
                q = (l >= 64) ? 0 : (apfx::wide_t)(int64_t)((uint64_t)raw << l);
            } else {
                const apfx::wide_t lim = (l >= 120) ? 0 : ((apfx::wide_t)1 << (120 - l));
                if (raw >= lim || raw <= -lim) q = (raw > 0) ? ((apfx::wide_t)1 << 100) : -((apfx::wide_t)1 << 100);
                else q = raw << l;
            }
        } else {
            q = raw;
        }
        return (raw_t)apfx::overflow<_AP_W, _AP_O>(q);
    }

    ap_fixed() : V(0) {}
    ap_fixed(const ap_fixed& o) = default;
    ap_fixed& operator=(const ap_fixed& o) = default;

    template <int W2, int I2, ap_q_mode Q2, ap_o_mode O2, int N2>
    ap_fixed(const ap_fixed<W2, I2, Q2, O2, N2>& o) : V(narrow((apfx::wide_t)o.V, W2 - I2)) {}

    ap_fixed(double d) { V = from_double(d); }
    ap_fixed(float f) { V = from_double((double)f); }
    ap_fixed(int i) : V(narrow((apfx::wide_t)i, 0)) {}
    ap_fixed(unsigned i) : V(narrow((apfx::wide_t)i, 0)) {}
    ap_fixed(long i) : V(narrow((apfx::wide_t)i, 0)) {}
    ap_fixed(unsigned long i) : V(narrow((apfx::wide_t)i, 0)) {}
    ap_fixed(long long i) : V(narrow((apfx::wide_t)i, 0)) {}
    ap_fixed(unsigned long long i) : V(narrow((apfx::wide_t)i, 0)) {}

    static raw_t from_double(double d) {
        if (std::isnan(d)) return 0;
        if (std::isinf(d)) {
            const apfx::wide_t big = (apfx::wide_t)1 << 100;
            return (raw_t)apfx::overflow<_AP_W, _AP_O>((_AP_O == AP_WRAP) ? 0 : (d > 0 ? big : -big));
        }
        if (d == 0.0) return 0;
        int ex = 0;
        const double fr = std::frexp(d, &ex);           // d = fr * 2^ex, 0.5 <= |fr| < 1
        const int64_t m = (int64_t)std::ldexp(fr, 53);  // exact 54-bit signed integer
        // d = m * 2^(ex-53); in destination raw units: m * 2^(ex-53+F)
        return narrow((apfx::wide_t)m, 53 - ex);
    }

    static ap_fixed from_raw(int64_t r) { ap_fixed x; x.V = (raw_t)r; return x; }

    double to_double() const { return std::ldexp((double)(int64_t)V, -F); }
    float to_float() const { return std::ldexp((float)(int64_t)V, -F); }
    explicit operator double() const { return to_double(); }
    explicit operator float() const { return to_float(); }

    // Compound assignment: exact result, then narrowed into this type.
    template <int W2, int I2, ap_q_mode Q2, ap_o_mode O2, int N2>
    ap_fixed& operator+=(const ap_fixed<W2, I2, Q2, O2, N2>& o) {
        const int fm = apfx::imax(F, W2 - I2);
        const apfx::wide_t a = (apfx::wide_t)V << (fm - F);
        const apfx::wide_t b = (apfx::wide_t)o.V << (fm - (W2 - I2));
        V = narrow(a + b, fm);
        return *this;
    }
    template <int W2, int I2, ap_q_mode Q2, ap_o_mode O2, int N2>
    ap_fixed& operator-=(const ap_fixed<W2, I2, Q2, O2, N2>& o) {
        const int fm = apfx::imax(F, W2 - I2);
        const apfx::wide_t a = (apfx::wide_t)V << (fm - F);
        const apfx::wide_t b = (apfx::wide_t)o.V << (fm - (W2 - I2));
        V = narrow(a - b, fm);
        return *this;
    }
    template <int W2, int I2, ap_q_mode Q2, ap_o_mode O2, int N2>
    ap_fixed& operator*=(const ap_fixed<W2, I2, Q2, O2, N2>& o) {
        V = narrow((apfx::wide_t)V * (apfx::wide_t)o.V, F + (W2 - I2));
        return *this;
    }
    ap_fixed& operator+=(double d) { return *this += ap_fixed<64, 32>(d); }
    ap_fixed& operator-=(double d) { return *this -= ap_fixed<64, 32>(d); }
};

// ---- full-precision binary arithmetic --------------------------------------

template <int W1, int I1, ap_q_mode Q1, ap_o_mode O1, int N1,
          int W2, int I2, ap_q_mode Q2, ap_o_mode O2, int N2>
inline ap_fixed<apfx::imax(I1, I2) + 1 + apfx::imax(W1 - I1, W2 - I2), apfx::imax(I1, I2) + 1>
operator+(const ap_fixed<W1, I1, Q1, O1, N1>& a, const ap_fixed<W2, I2, Q2, O2, N2>& b) {
    typedef ap_fixed<apfx::imax(I1, I2) + 1 + apfx::imax(W1 - I1, W2 - I2), apfx::imax(I1, I2) + 1> R;
    const int fm = R::F;
    const apfx::wide_t s = ((apfx::wide_t)a.V << (fm - (W1 - I1))) + ((apfx::wide_t)b.V << (fm - (W2 - I2)));
    return R::from_raw((int64_t)s);
}

template <int W1, int I1, ap_q_mode Q1, ap_o_mode O1, int N1,
          int W2, int I2, ap_q_mode Q2, ap_o_mode O2, int N2>
inline ap_fixed<apfx::imax(I1, I2) + 1 + apfx::imax(W1 - I1, W2 - I2), apfx::imax(I1, I2) + 1>
operator-(const ap_fixed<W1, I1, Q1, O1, N1>& a, const ap_fixed<W2, I2, Q2, O2, N2>& b) {
    typedef ap_fixed<apfx::imax(I1, I2) + 1 + apfx::imax(W1 - I1, W2 - I2), apfx::imax(I1, I2) + 1> R;
    const int fm = R::F;
    const apfx::wide_t s = ((apfx::wide_t)a.V << (fm - (W1 - I1))) - ((apfx::wide_t)b.V << (fm - (W2 - I2)));
    return R::from_raw((int64_t)s);
}

template <int W1, int I1, ap_q_mode Q1, ap_o_mode O1, int N1,
          int W2, int I2, ap_q_mode Q2, ap_o_mode O2, int N2>
inline ap_fixed<W1 + W2, I1 + I2>
operator*(const ap_fixed<W1, I1, Q1, O1, N1>& a, const ap_fixed<W2, I2, Q2, O2, N2>& b) {
    typedef ap_fixed<W1 + W2, I1 + I2> R;
    return R::from_raw((int64_t)((apfx::wide_t)a.V * (apfx::wide_t)b.V));
}

// Quotient keeps the dividend's fractional bits; the divisor's fractional bits
// are pre-shifted into the dividend; C integer division truncates toward zero.
// A zero divisor yields 0 here (the reference kernels guard it before dividing).
template <int W1, int I1, ap_q_mode Q1, ap_o_mode O1, int N1,
          int W2, int I2, ap_q_mode Q2, ap_o_mode O2, int N2>
inline ap_fixed<W1 + apfx::imax(W2 - I2, 0) + 1, I1 + (W2 - I2) + 1>
operator/(const ap_fixed<W1, I1, Q1, O1, N1>& a, const ap_fixed<W2, I2, Q2, O2, N2>& b) {
    typedef ap_fixed<W1 + apfx::imax(W2 - I2, 0) + 1, I1 + (W2 - I2) + 1> R;
    if (b.V == 0) return R::from_raw(0);
    const apfx::wide_t num = (apfx::wide_t)a.V << apfx::imax(W2 - I2, 0);
    return R::from_raw((int64_t)(num / (apfx::wide_t)b.V));
}

template <int W, int I, ap_q_mode Q, ap_o_mode O, int N>
inline ap_fixed<W + 1, I + 1> operator-(const ap_fixed<W, I, Q, O, N>& a) {
    return ap_fixed<W + 1, I + 1>::from_raw(-(int64_t)a.V);
}

// ---- comparisons (exact) ----------------------------------------------------

#define APFX_CMP(OP)                                                                    \
    template <int W1, int I1, ap_q_mode Q1, ap_o_mode O1, int N1,                       \
              int W2, int I2, ap_q_mode Q2, ap_o_mode O2, int N2>                       \
    inline bool operator OP(const ap_fixed<W1, I1, Q1, O1, N1>& a,                      \
                            const ap_fixed<W2, I2, Q2, O2, N2>& b) {                    \
        const int fm = apfx::imax(W1 - I1, W2 - I2);                                    \
        return ((apfx::wide_t)a.V << (fm - (W1 - I1))) OP((apfx::wide_t)b.V << (fm - (W2 - I2))); \
    }
APFX_CMP(==)
APFX_CMP(!=)
APFX_CMP(<)
APFX_CMP(<=)
APFX_CMP(>)
APFX_CMP(>=)
#undef APFX_CMP
