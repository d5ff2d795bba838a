// Element arithmetic shared by the INT8 quant kernels and the fused w13
// epilogue: SiLU*up rounded through the storage type, the tile absmax and the
// round-half-away INT8 quantisation, each with an exact fallback for the
// values a fast evaluation could round differently (reference
// int8_hybrid_moe/quant.py:195-209, 495-511).
#pragma once

#include <type_traits>

#include "common.cuh"

namespace i8moe {
namespace {

__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  return (static_cast<uint64_t>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }

__device__ __forceinline__ int8_t quant_exact(float x, float scale) {
  float v = __fdiv_rn(x, scale);
  v = fminf(fmaxf(v, -128.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(roundf(v)));
}

// |x|-max of one 16-byte chunk (NaN-ignoring).
template <typename T>
__device__ __forceinline__ float chunk_absmax(const uint4& v) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
    __nv_bfloat162 m2 = __hmax2(__habs2(h[0]), __habs2(h[1]));
    m2 = __hmax2(m2, __hmax2(__habs2(h[2]), __habs2(h[3])));
    return fmaxf(__low2float(m2), __high2float(m2));
  } else if constexpr (std::is_same<T, __half>::value) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
    __half2 m2 = __hmax2(__habs2(h[0]), __habs2(h[1]));
    m2 = __hmax2(m2, __hmax2(__habs2(h[2]), __habs2(h[3])));
    return fmaxf(__low2float(m2), __high2float(m2));
  } else {
    const float* f = reinterpret_cast<const float*>(&v);
    return fmaxf(fmaxf(fabsf(f[0]), fabsf(f[1])), fmaxf(fabsf(f[2]), fabsf(f[3])));
  }
}

// Exact SiLU of one chunk (the IEEE quotient for every element).
template <typename T>
__device__ __noinline__ uint4 silu_mul_chunk_exact(uint4 g, uint4 u) {
  constexpr int EPC = 16 / sizeof(T);
  uint4 o;
#pragma unroll
  for (int i = 0; i < EPC; ++i) {
    const float gf = Num<T>::to_f(reinterpret_cast<const T*>(&g)[i]);
    const float uf = Num<T>::to_f(reinterpret_cast<const T*>(&u)[i]);
    const float sn = Num<T>::to_f(Num<T>::from_f(__fdiv_rn(gf, 1.0f + expf(-gf))));
    reinterpret_cast<T*>(&o)[i] = Num<T>::from_f(sn * uf);
  }
  return o;
}

// act = dtype(dtype(g / (1 + exp(-g))) * up) for one chunk.  The quotient is
// evaluated as g * rcp(1 + exp(-g)) (__fdividef), within 2.5 ulp of the IEEE
// quotient while the divisor stays below 2^126.  For g < -80 the divisor
// (>= e^80 ~ 2^115, infinite past -88.72) is first scaled by 2^-64 and the
// quotient scaled back -- both exact power-of-two steps -- so the same bound
// holds down to the overflow of exp, where both evaluations give -0.  For
// large positive g the divisor rounds to 1 and the quotient is exact.  The
// 16-bit rounding of the two quotients therefore agrees unless the value lies
// within 4 ulp of a rounding midpoint of the storage type (or, in the fp16
// subnormal range, within 4e-4 quanta of one); such chunks are recomputed
// with the IEEE division.
template <typename T>
__device__ __forceinline__ uint4 silu_mul_chunk(const uint4& g, const uint4& u) {
  if constexpr (sizeof(T) == 4) {
    return silu_mul_chunk_exact<T>(g, u);
  } else {
    constexpr int EPC = 8;
    const float kDown = __int_as_float(0x1F800000);  // 2^-64
    uint4 o;
    bool need = false;
#pragma unroll
    for (int i = 0; i < EPC; ++i) {
      const float gf = Num<T>::to_f(reinterpret_cast<const T*>(&g)[i]);
      const float uf = Num<T>::to_f(reinterpret_cast<const T*>(&u)[i]);
      const float den = 1.0f + expf(-gf);
      const float y = gf < -80.0f ? __fdividef(gf, den * kDown) * kDown : __fdividef(gf, den);
      const uint32_t b = __float_as_uint(y);
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        need |= (((b + 4u) & 0xFFFFu) - 0x8000u) <= 8u;
      } else {
        const float ay = fabsf(y);
        if (ay < 6.103515625e-05f) {  // fp16 subnormal: quantum 2^-24
          const float t = ay * 16777216.0f;
          need |= fabsf((t - floorf(t)) - 0.5f) < 4.0e-4f;
        } else {
          need |= (((b + 4u) & 0x1FFFu) - 0x1000u) <= 8u;
        }
      }
      const float sn = Num<T>::to_f(Num<T>::from_f(y));
      reinterpret_cast<T*>(&o)[i] = Num<T>::from_f(sn * uf);
    }
    if (need) o = silu_mul_chunk_exact<T>(g, u);
    return o;
  }
}

// Fast INT8 quantisation of one chunk: x * inv (packed f32x2), rounded by the
// 1.5*2^23 trick; returns false when an element lies within 3e-5 of a
// rounding tie (or is not finite) so the caller takes the exact path.
template <typename T>
__device__ __forceinline__ bool quant_chunk_fast(const uint4& v, float inv,
                                                 uint32_t (&words)[16 / sizeof(T) / 4]) {
  constexpr int EPC = 16 / sizeof(T);
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const uint64_t inv2 = f2_pack(inv, inv);
  const uint64_t magic2 = f2_pack(kMagic, kMagic);
  const uint64_t nmagic2 = f2_pack(-kMagic, -kMagic);
  float dmax = 0.0f;
#pragma unroll
  for (int w = 0; w < EPC / 4; ++w) {
    float f[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = Num<T>::to_f(reinterpret_cast<const T*>(&v)[4 * w + i]);
    const uint64_t y01 = f2_mul(f2_pack(f[0], f[1]), inv2);
    const uint64_t y23 = f2_mul(f2_pack(f[2], f[3]), inv2);
    const uint64_t t01 = f2_add(y01, magic2);
    const uint64_t t23 = f2_add(y23, magic2);
    // d = y - rint(y): t - 1.5*2^23 is exact, negated by flipping the signs
    const uint64_t d01 = f2_add(y01, f2_add(t01, nmagic2) ^ 0x8000000080000000ull);
    const uint64_t d23 = f2_add(y23, f2_add(t23, nmagic2) ^ 0x8000000080000000ull);
    dmax = max_nan(dmax, fabsf(f2_lo(d01)));
    dmax = max_nan(dmax, fabsf(f2_hi(d01)));
    dmax = max_nan(dmax, fabsf(f2_lo(d23)));
    dmax = max_nan(dmax, fabsf(f2_hi(d23)));
    const uint32_t lo = __byte_perm(static_cast<uint32_t>(t01), static_cast<uint32_t>(t01 >> 32), 0x0040);
    const uint32_t hi = __byte_perm(static_cast<uint32_t>(t23), static_cast<uint32_t>(t23 >> 32), 0x0040);
    words[w] = __byte_perm(lo, hi, 0x5410);
  }
  return dmax < 0.49997f;
}

// ---------------------------------------------------------------------------
// Bracketed INT8 quantisation of 16-bit chunks.
//
// With inv = RN(1/scale), inv_lo = RD(inv * (1 - 2^-20)) and
// inv_hi = RU(inv * (1 + 2^-20)), the IEEE quotient RN(x / scale) lies
// strictly between x * inv_lo and x * inv_hi (the reciprocal and the
// quotient are each within 2^-24 relative of exact, far inside the 2^-20
// margin).  Both products are rounded to an integer by one FMA each
// (fma(x, inv, 1.5 * 2^23): round to nearest even, the integer in the low
// bits of the result).  Rounding is monotonic, so when the two integers agree
// every value between them -- the quotient included -- rounds to that integer,
// and the quotient is not an exact tie (a tie k + 0.5 strictly inside the
// bracket would round the ends to k and k + 1), so round-half-away equals
// round-to-nearest-even there.  Agreement is tested for a whole chunk at once:
// s += (t_lo - t_hi)^2 stays 0 exactly when every pair agrees and no value is
// NaN or infinite; otherwise the chunk is recomputed with the IEEE division.
// |x / scale| <= 127 (1 + 2^-23) because |x| <= the tile absmax, so no clamp
// binds on the fast path.  Packed f32x2 arithmetic throughout.
// ---------------------------------------------------------------------------
struct QuantInv {
  float lo, hi;
};

__device__ __forceinline__ QuantInv quant_inv(float scale) {
  const float inv = __frcp_rn(scale);
  return QuantInv{__fmul_rd(inv, 1.0f - 0x1p-20f), __fmul_ru(inv, 1.0f + 0x1p-20f)};
}

__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// Fast path for one 8-element chunk of bf16 / fp16: the eight int8 values in
// out; false if the chunk needs the exact path.  Each 32-bit word (two
// values) goes through one asm block: unpack to an f32x2 pair, the two
// bracketing FMAs, the agreement sum and the byte extraction, with the pairs
// built by mov.b64 inside the block.
template <typename T>
__device__ __forceinline__ bool quant_chunk_bracket(const uint4& v, const QuantInv& qi,
                                                    uint2& out) {
  static_assert(sizeof(T) == 2, "16-bit activations");
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const uint64_t lo2 = f2_pack(qi.lo, qi.lo), hi2 = f2_pack(qi.hi, qi.hi);
  const uint64_t m2 = f2_pack(kMagic, kMagic);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t b[4];
  uint64_t s = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // b[i]: the low byte of each lane's integer, lanes 0 and 1 in bytes 0, 1
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      asm("{\n\t.reg .b32 x0, x1, a0, a1;\n\t.reg .b64 x, ta, tb, dd;\n\t"
          "shl.b32 x0, %2, 16;\n\t"
          "and.b32 x1, %2, 0xFFFF0000;\n\t"
          "mov.b64 x, {x0, x1};\n\t"
          "fma.rn.f32x2 ta, x, %3, %5;\n\t"
          "fma.rn.f32x2 tb, x, %4, %5;\n\t"
          "sub.rn.f32x2 dd, ta, tb;\n\t"
          "fma.rn.f32x2 %1, dd, dd, %1;\n\t"
          "mov.b64 {a0, a1}, ta;\n\t"
          "prmt.b32 %0, a0, a1, 0x0040;\n\t}"
          : "=r"(b[i]), "+l"(s)
          : "r"(w[i]), "l"(lo2), "l"(hi2), "l"(m2));
    } else {
      asm("{\n\t.reg .b16 h0, h1;\n\t.reg .b32 x0, x1, a0, a1;\n\t.reg .b64 x, ta, tb, dd;\n\t"
          "mov.b32 {h0, h1}, %2;\n\t"
          "cvt.f32.f16 x0, h0;\n\t"
          "cvt.f32.f16 x1, h1;\n\t"
          "mov.b64 x, {x0, x1};\n\t"
          "fma.rn.f32x2 ta, x, %3, %5;\n\t"
          "fma.rn.f32x2 tb, x, %4, %5;\n\t"
          "sub.rn.f32x2 dd, ta, tb;\n\t"
          "fma.rn.f32x2 %1, dd, dd, %1;\n\t"
          "mov.b64 {a0, a1}, ta;\n\t"
          "prmt.b32 %0, a0, a1, 0x0040;\n\t}"
          : "=r"(b[i]), "+l"(s)
          : "r"(w[i]), "l"(lo2), "l"(hi2), "l"(m2));
    }
  }
  out.x = __byte_perm(b[0], b[1], 0x5410);
  out.y = __byte_perm(b[2], b[3], 0x5410);
  return (static_cast<uint32_t>(s) | static_cast<uint32_t>(s >> 32)) == 0u;
}

// Exact reference rounding of one 8-element 16-bit chunk, returned by value.
template <typename T>
__device__ __noinline__ uint2 quant_chunk_exact16(uint4 v, float scale) {
  uint32_t q[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    q[i] = static_cast<uint8_t>(quant_exact(Num<T>::to_f(reinterpret_cast<const T*>(&v)[i]), scale));
  return make_uint2(q[0] | (q[1] << 8) | (q[2] << 16) | (q[3] << 24),
                    q[4] | (q[5] << 8) | (q[6] << 16) | (q[7] << 24));
}

// Running |x|-max of 16-bit chunks as a packed pair (NaN-ignoring, as fmaxf):
// acc starts at 0; absmax16_value gives the float maximum.
template <typename T>
__device__ __forceinline__ uint32_t absmax16_acc(uint32_t acc, const uint4& v) {
  uint32_t r = acc;
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value)
      asm("max.xorsign.abs.bf16x2 %0, %0, %1;" : "+r"(r) : "r"(w[i]));
    else
      asm("max.xorsign.abs.f16x2 %0, %0, %1;" : "+r"(r) : "r"(w[i]));
  }
  return r;
}
template <typename T>
__device__ __forceinline__ float absmax16_value(uint32_t acc) {
  acc &= 0x7FFF7FFFu;  // the xorsign form leaves a sign bit
  const T* h = reinterpret_cast<const T*>(&acc);
  return fmaxf(Num<T>::to_f(h[0]), Num<T>::to_f(h[1]));
}

// Exact reference rounding for one chunk: round_half_away(clamp(x / scale)).
template <typename T>
__device__ __noinline__ void quant_chunk_exact(uint4 v, float inv, float scale,
                                               uint32_t (&words)[16 / sizeof(T) / 4]) {
  constexpr int EPC = 16 / sizeof(T);
  constexpr float kMagic = 12582912.0f;
#pragma unroll
  for (int i = 0; i < EPC; ++i) {
    const float x = Num<T>::to_f(reinterpret_cast<const T*>(&v)[i]);
    const float y = __fmul_rn(x, inv);
    const float d = fabsf(y - (__fadd_rn(y, kMagic) - kMagic));
    if (!(d < 0.49997f)) {
      const uint32_t q = static_cast<uint8_t>(quant_exact(x, scale));
      words[i / 4] = (words[i / 4] & ~(0xFFu << (8 * (i % 4)))) | (q << (8 * (i % 4)));
    }
  }
}

// As quant_chunk_exact, with ties rounded to even (torch.round / rint), for the
// weight preparation: clamp(rint(x / scale)).
template <typename T>
__device__ __noinline__ void quant_chunk_exact_rne(uint4 v, float scale,
                                                   uint32_t (&words)[16 / sizeof(T) / 4]) {
  constexpr int EPC = 16 / sizeof(T);
#pragma unroll
  for (int i = 0; i < EPC; ++i) {
    const float x = Num<T>::to_f(reinterpret_cast<const T*>(&v)[i]);
    const float q = fminf(fmaxf(rintf(__fdiv_rn(x, scale)), -128.0f), 127.0f);
    const uint32_t b = static_cast<uint8_t>(static_cast<int8_t>(static_cast<int>(q)));
    words[i / 4] = (words[i / 4] & ~(0xFFu << (8 * (i % 4)))) | (b << (8 * (i % 4)));
  }
}

}  // namespace
}  // namespace i8moe
