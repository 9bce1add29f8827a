// Shared device helpers for the sm_100a kernels of libms_engine.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ms {

constexpr int kWarp = 32;
constexpr unsigned kFull = 0xffffffffu;

// ---- element conversion ----------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};

// Round an f32 value to the storage type and back (the "cast to model dtype"
// points of the reference's Candle ops).
template <typename T> __device__ __forceinline__ float round_to(float v) {
  return Elem<T>::to_f(Elem<T>::from_f(v));
}

// Load / store 4 consecutive elements as f32.
template <typename T> struct Vec4;
template <> struct Vec4<float> {
  static __device__ __forceinline__ void load(const float *p, float (&o)[4]) {
    float4 v = *reinterpret_cast<const float4 *>(p);
    o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
  }
  static __device__ __forceinline__ void store(float *p, const float (&o)[4]) {
    *reinterpret_cast<float4 *>(p) = make_float4(o[0], o[1], o[2], o[3]);
  }
};
template <> struct Vec4<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16 *p, float (&o)[4]) {
    uint2 u = *reinterpret_cast<const uint2 *>(p);
    o[0] = __uint_as_float(u.x << 16); o[1] = __uint_as_float(u.x & 0xffff0000u);
    o[2] = __uint_as_float(u.y << 16); o[3] = __uint_as_float(u.y & 0xffff0000u);
  }
  static __device__ __forceinline__ void store(__nv_bfloat16 *p, const float (&o)[4]) {
    __nv_bfloat162 a = __floats2bfloat162_rn(o[0], o[1]);
    __nv_bfloat162 b = __floats2bfloat162_rn(o[2], o[3]);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t *>(&a);
    u.y = *reinterpret_cast<uint32_t *>(&b);
    *reinterpret_cast<uint2 *>(p) = u;
  }
};
template <> struct Vec4<__half> {
  static __device__ __forceinline__ void load(const __half *p, float (&o)[4]) {
    uint2 u = *reinterpret_cast<const uint2 *>(p);
    __half2 a = *reinterpret_cast<__half2 *>(&u.x);
    __half2 b = *reinterpret_cast<__half2 *>(&u.y);
    float2 fa = __half22float2(a), fb = __half22float2(b);
    o[0] = fa.x; o[1] = fa.y; o[2] = fb.x; o[3] = fb.y;
  }
  static __device__ __forceinline__ void store(__half *p, const float (&o)[4]) {
    __half2 a = __floats2half2_rn(o[0], o[1]);
    __half2 b = __floats2half2_rn(o[2], o[3]);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t *>(&a);
    u.y = *reinterpret_cast<uint32_t *>(&b);
    *reinterpret_cast<uint2 *>(p) = u;
  }
};

// Load / store 2 consecutive elements as f32.
template <typename T> struct Vec2;
template <> struct Vec2<float> {
  static __device__ __forceinline__ void load(const float *p, float (&o)[2]) {
    float2 v = *reinterpret_cast<const float2 *>(p);
    o[0] = v.x; o[1] = v.y;
  }
  static __device__ __forceinline__ void store(float *p, const float (&o)[2]) {
    *reinterpret_cast<float2 *>(p) = make_float2(o[0], o[1]);
  }
};
template <> struct Vec2<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16 *p, float (&o)[2]) {
    uint32_t u = *reinterpret_cast<const uint32_t *>(p);
    o[0] = __uint_as_float(u << 16); o[1] = __uint_as_float(u & 0xffff0000u);
  }
  static __device__ __forceinline__ void store(__nv_bfloat16 *p, const float (&o)[2]) {
    *reinterpret_cast<__nv_bfloat162 *>(p) = __floats2bfloat162_rn(o[0], o[1]);
  }
};
template <> struct Vec2<__half> {
  static __device__ __forceinline__ void load(const __half *p, float (&o)[2]) {
    float2 f = __half22float2(*reinterpret_cast<const __half2 *>(p));
    o[0] = f.x; o[1] = f.y;
  }
  static __device__ __forceinline__ void store(__half *p, const float (&o)[2]) {
    *reinterpret_cast<__half2 *>(p) = __floats2half2_rn(o[0], o[1]);
  }
};

// ---- 16 bytes of T kept as raw bits (one vector load / store) ----------------
// Values that are already representable in T (sums rounded to the model dtype)
// stay packed in registers at half the cost of f32 copies for 16-bit T.
template <typename T> struct Raw16;
template <> struct Raw16<float> {
  static constexpr int N = 4;
  static __device__ __forceinline__ void unpack(const uint4 &v, float (&o)[4]) {
    o[0] = __uint_as_float(v.x); o[1] = __uint_as_float(v.y);
    o[2] = __uint_as_float(v.z); o[3] = __uint_as_float(v.w);
  }
  static __device__ __forceinline__ uint4 pack(const float (&o)[4]) {
    return make_uint4(__float_as_uint(o[0]), __float_as_uint(o[1]), __float_as_uint(o[2]), __float_as_uint(o[3]));
  }
};
template <> struct Raw16<__nv_bfloat16> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void unpack(const uint4 &v, float (&o)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      o[2 * k] = __uint_as_float(w[k] << 16);
      o[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
    }
  }
  static __device__ __forceinline__ uint4 pack(const float (&o)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      __nv_bfloat162 h = __floats2bfloat162_rn(o[2 * k], o[2 * k + 1]);
      w[k] = *reinterpret_cast<uint32_t *>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};
template <> struct Raw16<__half> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void unpack(const uint4 &v, float (&o)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[k]));
      o[2 * k] = f.x;
      o[2 * k + 1] = f.y;
    }
  }
  static __device__ __forceinline__ uint4 pack(const float (&o)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      __half2 h = __floats2half2_rn(o[2 * k], o[2 * k + 1]);
      w[k] = *reinterpret_cast<uint32_t *>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};

__device__ __forceinline__ bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// ---- x / n for many x and one n ----------------------------------------------
// Markstein's correction (P. Markstein, "Computation of elementary functions
// on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990): with
// r = RN(1/n) and q0 = RN(x * r), the residual e = x - n * q0 is exact in one
// FMA and RN(q0 + e * r) is the correctly rounded quotient RN(x / n) for
// normal operands.  Callers compute r = 1.0f / n once (an IEEE division) and
// pay two FMAs and a multiply per element instead of a full division.
__device__ __forceinline__ float div_by(float x, float n, float r) {
  const float q0 = x * r;
  const float e = fmaf(-q0, n, x);
  return fmaf(e, r, q0);
}

// ---- packed bf16x2 arithmetic on raw 32-bit words ----------------------------
// For bf16 operands a product is exact in f32 and a sum is either exact in f32
// or differs from the larger operand by far less than half a bf16 ulp, so
// round_to<bf16>(float(a) op float(b)) equals the correctly rounded bf16x2
// result of the hardware instruction: one instruction per two values and no
// f32 -> bf16 conversion.
__device__ __forceinline__ uint32_t bf2_mul(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hmul2(*reinterpret_cast<const __nv_bfloat162 *>(&a), *reinterpret_cast<const __nv_bfloat162 *>(&b));
  return *reinterpret_cast<uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t bf2_add(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hadd2(*reinterpret_cast<const __nv_bfloat162 *>(&a), *reinterpret_cast<const __nv_bfloat162 *>(&b));
  return *reinterpret_cast<uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t bf2_pack(float lo, float hi) {
  __nv_bfloat162 r = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&r);
}
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ uint32_t u4_get(const uint4 &v, int k) { return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w; }
__device__ __forceinline__ void u4_set(uint4 &v, int k, uint32_t w) {
  if (k == 0) v.x = w; else if (k == 1) v.y = w; else if (k == 2) v.z = w; else v.w = w;
}

// ---- packed f32x2 arithmetic (sm_100: two f32 lanes per instruction) ---------
// (d0, d1) = (a0, a1) * b + c, one packed f32x2 FMA (each lane rounded once, as fmaf)
__device__ __forceinline__ void ffma2(float &d0, float &d1, float a0, float a1, float b, float c) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %4};\n\t"
      "mov.b64 rc, {%5, %5};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b), "f"(c));
}
// (d0, d1) += (a0, a1), one packed f32x2 add
__device__ __forceinline__ void fadd2(float &d0, float &d1, float a0, float a1) {
  asm("{\n\t.reg .b64 ra, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rd, {%0, %1};\n\t"
      "add.rn.f32x2 rd, rd, ra;\n\tmov.b64 {%0, %1}, rd;\n}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1));
}
// (d0, d1) = (a0, a1) + (b0, b1) and (d0, d1) = (a0, a1) * (b0, b1) + (c0, c1), packed f32x2
__device__ __forceinline__ void add2(float &d0, float &d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
__device__ __forceinline__ void fma2(float &d0, float &d1, float a0, float a1, float b0, float b1, float c0,
                                     float c1) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
// (d0, d1) = (a0, a1) * (b0, b1), packed f32x2
__device__ __forceinline__ void mul2(float &d0, float &d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// ---- warp reductions ---------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
  return v;
}

// Device-side status word: kernels record a problem here instead of faulting.
// Bits: 1 = mbarrier wait gave up, 2 = index out of range.
constexpr unsigned kStatusWaitTimeout = 1u;
constexpr unsigned kStatusBadIndex = 2u;

}  // namespace ms
