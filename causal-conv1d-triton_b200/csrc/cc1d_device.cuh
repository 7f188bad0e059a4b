// Device-side building blocks shared by every kernel of the causal depthwise conv1d path:
// dtype codes, mbarrier / TMA wrappers (inline PTX for sm_100a), bounded waits that report a
// status word instead of hanging, packed f32x2 arithmetic, and vector load/convert/store helpers.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

namespace cc1d {

// Element type codes used across the C ABI (include/causal_conv1d_b200.h).
enum : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

// Bits of the device status word (read back with cc1d_status()).
enum : unsigned { kStatusWaitTimeout = 1u };

// Every wait on an mbarrier gives up after this long, records kStatusWaitTimeout and returns.
constexpr unsigned long long kWaitLimitNs = 1000000000ull;  // 1 s

// Calls f(std::integral_constant<int, I>{}) for I = B .. E-1 in order. Unlike `#pragma unroll`,
// the body is always instantiated once per index, so arrays indexed by I stay in registers with
// fixed assignments (a ring indexed by (I + k) % N moves no values).
template <int B, int E, typename F>
__device__ __forceinline__ void static_for(F&& f) {
  if constexpr (B < E) {
    f(std::integral_constant<int, B>{});
    static_for<B + 1, E>(f);
  }
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// The first ALIGN-aligned byte of a dynamic shared-memory array, as an offset from the array
// itself: rounding the address up through an integer would hide from the compiler that the
// result points into shared memory, and the loads and stores through it would be issued as
// generic accesses instead of shared-memory ones.
template <int ALIGN>
__device__ __forceinline__ unsigned char* aligned_smem(unsigned char* raw) {
  const uint32_t a = smem_u32(raw);
  return raw + (((a + (ALIGN - 1)) & ~uint32_t(ALIGN - 1)) - a);
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes the initialised barriers visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Adds `bytes` to the transaction count of the current phase without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete. Returns false (and records a timeout in
// *status) if it has not completed within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      atomicOr(status, kStatusWaitTimeout);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------------------------
// TMA
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 3-D tiled bulk tensor load global -> shared, completion counted on `bar` in bytes.
// c0 is the innermost (channel) coordinate and must be a multiple of 16 bytes; c1 (time) may be
// negative or past the end, where the box is zero-filled.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// Register budget changes of a warpgroup (every thread of its four warps executes the same one):
// dec releases registers to the SM sub-partition, inc waits until it can take them.
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// Named barrier over the first `nthreads` threads (warp multiples) of the CTA.
__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------------------------
// Packed fp32 pair arithmetic (sm_100 f32x2 instructions): two lanes of fp32 per instruction,
// each lane rounded exactly as the scalar operation would be.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) { return __fadd2_rn(a, b); }

// tanh.approx.f32 (one MUFU op). Max relative error about 2^-11.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Logistic sigmoid of a pair. FAST uses sigmoid(z) = 0.5 + 0.5 tanh(z / 2) with the one-op
// hardware tanh (used when the result is rounded to a 16-bit type); otherwise
// 1 / (1 + exp(-z)) with the exp and divide intrinsics, accurate to a few fp32 ulp.
template <bool FAST>
__device__ __forceinline__ float2 sigmoid2(float2 z) {
  if constexpr (FAST) {
    const float2 h = fmul2(z, make_float2(0.5f, 0.5f));
    const float2 t = make_float2(tanh_approx(h.x), tanh_approx(h.y));
    return ffma2(t, make_float2(0.5f, 0.5f), make_float2(0.5f, 0.5f));
  } else {
    return make_float2(__fdividef(1.0f, 1.0f + __expf(-z.x)), __fdividef(1.0f, 1.0f + __expf(-z.y)));
  }
}

// SiLU of a pair, z * sigmoid(z). FAST writes it as h + h * tanh(h) with h = z / 2 (one MUFU op
// per element); otherwise z times the accurate sigmoid above.
template <bool FAST>
__device__ __forceinline__ float2 silu2(float2 z) {
  if constexpr (FAST) {
    const float2 h = fmul2(z, make_float2(0.5f, 0.5f));
    const float2 t = make_float2(tanh_approx(h.x), tanh_approx(h.y));
    return ffma2(h, t, h);
  } else {
    return fmul2(z, sigmoid2<false>(z));
  }
}

// The 16-bit (FAST) SiLU paths run on h = z / 2 directly: the kernels scale their fp32 taps and
// bias by 0.5 once, which is exact in binary floating point, so the convolution yields h with the
// bits of 0.5 * z. With t = tanh(h):
//   SiLU(z)        = h + h t
//   2 SiLU'(z)     = 1 + t + h (1 - t^2)      (= 2 sig (1 + z (1 - sig)), sig = (1 + t) / 2)
// The backward multiplies dy by 2 SiLU'(z); the halved taps turn that back into dx exactly.
__device__ __forceinline__ float2 tanh2(float2 h) { return make_float2(tanh_approx(h.x), tanh_approx(h.y)); }

__device__ __forceinline__ float2 silu2_of_half(float2 h) { return ffma2(h, tanh2(h), h); }

// dy * 2 SiLU'(z) from h = z / 2, in three multiply-adds: 1 + t + h (1 - t^2) factors as
// (1 + t) (1 + h (1 - t)).
__device__ __forceinline__ float2 dsilu2_of_half(float2 h, float2 dy) {
  const float2 t = tanh2(h);
  const float2 g = ffma2(dy, t, dy);                      // dy (1 + t)
  const float2 e = ffma2(h, make_float2(-t.x, -t.y), h);  // h (1 - t)
  return ffma2(g, e, g);
}

// ---------------------------------------------------------------------------------------------
// cp.async (8-byte chunks) with completion counted on an mbarrier
// ---------------------------------------------------------------------------------------------
// Copies 8 bytes global -> shared; src_bytes = 0 writes zeros and reads nothing.
__device__ __forceinline__ void cp_async_8(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}

// One arrival on `bar` once every cp.async this thread issued before has completed (the arrival
// counts toward the barrier's expected count).
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// ---------------------------------------------------------------------------------------------
// Conversions
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float2 bf16x2_to_f2(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}
__device__ __forceinline__ uint32_t f2_to_bf16x2(float2 f) {
  __nv_bfloat162 h = __float22bfloat162_rn(f);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 f16x2_to_f2(uint32_t u) {
  return __half22float2(*reinterpret_cast<__half2*>(&u));
}
__device__ __forceinline__ uint32_t f2_to_f16x2(float2 f) {
  __half2 h = __float22half2_rn(f);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <typename T>
__device__ __forceinline__ float2 word_to_f2(uint32_t u) {
  if constexpr (std::is_same_v<T, __nv_bfloat16>)
    return bf16x2_to_f2(u);
  else
    return f16x2_to_f2(u);
}
template <typename T>
__device__ __forceinline__ uint32_t f2_to_word(float2 f) {
  if constexpr (std::is_same_v<T, __nv_bfloat16>)
    return f2_to_bf16x2(f);
  else
    return f2_to_f16x2(f);
}

// Loads CPT consecutive elements (CPT * sizeof(T) = 8 or 16 bytes, aligned to that) as fp32 pairs.
template <typename T, int CPT>
__device__ __forceinline__ void load_vec(const T* p, float2 (&v)[CPT / 2]) {
  constexpr int NW = CPT * static_cast<int>(sizeof(T)) / 4;
  static_assert(NW == 1 || NW == 2 || NW == 4, "4-, 8- or 16-byte vectors");
  uint32_t w[NW];
  if constexpr (NW == 4) {
    const uint4 q = *reinterpret_cast<const uint4*>(p);
    w[0] = q.x, w[1] = q.y, w[2] = q.z, w[3] = q.w;
  } else if constexpr (NW == 2) {
    const uint2 q = *reinterpret_cast<const uint2*>(p);
    w[0] = q.x, w[1] = q.y;
  } else {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < CPT / 2; ++i) v[i] = make_float2(__uint_as_float(w[2 * i]), __uint_as_float(w[2 * i + 1]));
  } else {
#pragma unroll
    for (int i = 0; i < CPT / 2; ++i) v[i] = word_to_f2<T>(w[i]);
  }
}

// Rounds CPT fp32 values to T (round to nearest even) and stores them as one vector.
template <typename T, int CPT>
__device__ __forceinline__ void store_vec(T* p, const float2 (&v)[CPT / 2]) {
  constexpr int NW = CPT * static_cast<int>(sizeof(T)) / 4;
  uint32_t w[NW];
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < CPT / 2; ++i) w[2 * i] = __float_as_uint(v[i].x), w[2 * i + 1] = __float_as_uint(v[i].y);
  } else {
#pragma unroll
    for (int i = 0; i < CPT / 2; ++i) w[i] = f2_to_word<T>(v[i]);
  }
  if constexpr (NW == 4)
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  else if constexpr (NW == 2)
    *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
  else
    *reinterpret_cast<uint32_t*>(p) = w[0];
}

// Scalar load of element `i` of a buffer whose element type is given at run time.
__device__ __forceinline__ float ld_any(const void* base, int64_t i, int dtype) {
  if (dtype == kF32) return static_cast<const float*>(base)[i];
  if (dtype == kBF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
  return __half2float(static_cast<const __half*>(base)[i]);
}

// Scalar store of element `i`, rounded to the run-time element type.
__device__ __forceinline__ void st_any(void* base, int64_t i, int dtype, float v) {
  if (dtype == kF32)
    static_cast<float*>(base)[i] = v;
  else if (dtype == kBF16)
    static_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
  else
    static_cast<__half*>(base)[i] = __float2half_rn(v);
}

template <typename T>
__device__ __forceinline__ float to_f(T v) {
  if constexpr (std::is_same_v<T, float>)
    return v;
  else if constexpr (std::is_same_v<T, __nv_bfloat16>)
    return __bfloat162float(v);
  else
    return __half2float(v);
}

template <typename T>
__device__ __forceinline__ T from_f(float v) {
  if constexpr (std::is_same_v<T, float>)
    return v;
  else if constexpr (std::is_same_v<T, __nv_bfloat16>)
    return __float2bfloat16_rn(v);
  else
    return __float2half_rn(v);
}

}  // namespace cc1d
