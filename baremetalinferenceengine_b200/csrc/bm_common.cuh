// Device helpers shared by the layer-op kernels: element types, 16-byte vector
// loads/stores with cache hints, warp reductions and device status bits.
//
// Every kernel computes in fp32. Storage is fp32 or bf16; a bf16 value widens to
// fp32 exactly (a 16-bit shift) and narrows with round-to-nearest-even.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "bm_layer_ops.h"

namespace bm {

using bf16 = __nv_bfloat16;

// Elements of T in one 16-byte vector.
template <typename T>
struct VecWidth;
template <>
struct VecWidth<float> {
  static constexpr int value = 4;
};
template <>
struct VecWidth<bf16> {
  static constexpr int value = 8;
};

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Two fp32 values to one word of two bf16 (lo in the low half), RNE.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

// 16 bytes of T -> VecWidth<T> floats.
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& v, float* f) {
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  } else {
    f[0] = bf16_lo(v.x);
    f[1] = bf16_hi(v.x);
    f[2] = bf16_lo(v.y);
    f[3] = bf16_hi(v.y);
    f[4] = bf16_lo(v.z);
    f[5] = bf16_hi(v.z);
    f[6] = bf16_lo(v.w);
    f[7] = bf16_hi(v.w);
  }
}

// VecWidth<T> floats -> 16 bytes of T.
template <typename T>
__device__ __forceinline__ uint4 pack16(const float* f) {
  uint4 v;
  if constexpr (sizeof(T) == 4) {
    v.x = __float_as_uint(f[0]);
    v.y = __float_as_uint(f[1]);
    v.z = __float_as_uint(f[2]);
    v.w = __float_as_uint(f[3]);
  } else {
    v.x = pack_bf16x2(f[0], f[1]);
    v.y = pack_bf16x2(f[2], f[3]);
    v.z = pack_bf16x2(f[4], f[5]);
    v.w = pack_bf16x2(f[6], f[7]);
  }
  return v;
}

// Rounds an fp32 value to the storage type and back (the value a store keeps).
template <typename T>
__device__ __forceinline__ float round_to(float x) {
  if constexpr (sizeof(T) == 4) {
    return x;
  } else {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
}

// Scalar element access.
template <typename T>
__device__ __forceinline__ float load1(const T* p) {
  if constexpr (sizeof(T) == 4) {
    return *reinterpret_cast<const float*>(p);
  } else {
    return __bfloat162float(*p);
  }
}
template <typename T>
__device__ __forceinline__ void store1(T* p, float x) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float*>(p) = x;
  } else {
    *p = __float2bfloat16_rn(x);
  }
}

// Streaming 16-byte load: read once, evict first (ld.global.cs). Coherent, so
// safe on buffers the same kernel writes (in-place ops).
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  return __ldcs(reinterpret_cast<const uint4*>(p));
}
// Read-only 16-byte load that should stay cached (weights, tables).
__device__ __forceinline__ uint4 ld_keep(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ void st_plain(void* p, const uint4& v) {
  *reinterpret_cast<uint4*>(p) = v;
}
__device__ __forceinline__ void st_stream(void* p, const uint4& v) {
  __stcs(reinterpret_cast<uint4*>(p), v);
}

// exp(-g) = 2^(-g * log2(e)) with the hardware's ex2.approx, and the reciprocal
// with rcp.approx (both single MUFU instructions; relative errors near 2^-22).
// ex2 of a large argument is +inf and rcp(+inf) is +0, so silu(-1000) = -0 and
// silu(+1000) = 1000 exactly as in the reference's known-answer test
// (tests/kernel_tests.cu:164-173).
__device__ __forceinline__ float silu_fast(float g) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(g * -1.4426950408889634f));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
  return g * r;
}

// One SwiGLU element, silu(g) * u (reference swiglu_kernel, src/kernels.cu:185-190):
// fp32 I/O computes g / (1 + expf(-g)) * u exactly as the reference writes it;
// bf16 I/O uses silu_fast, whose error is far below bf16 rounding.
template <typename T>
__device__ __forceinline__ float swiglu1(float g, float u) {
  if constexpr (sizeof(T) == 4) {
    return g / (1.0f + expf(-g)) * u;
  } else {
    return silu_fast(g) * u;
  }
}

// One RoPE pair, HF half-split (src/kernels.cu:131-139): element i and i + hd/2
// at angle (cos, sin) become (first cos - second sin, second cos + first sin).
// The roundings are spelled out (one product rounded, then one fused multiply-add)
// so the compiler cannot contract the expression differently in different
// kernels: every kernel that rotates calls this, and a fused form's results equal
// the RoPE kernels' bit for bit.
__device__ __forceinline__ void rope_rotate(float first, float second, float2 cs, float* o1, float* o2) {
  *o1 = __fmaf_rn(first, cs.x, -__fmul_rn(second, cs.y));
  *o2 = __fmaf_rn(second, cs.x, __fmul_rn(first, cs.y));
}

// Butterfly sum: every lane of the warp gets the total.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

__device__ __forceinline__ void raise_status(int32_t* status, int32_t bits) {
  if (status != nullptr) atomicOr(status, bits);
}

// First statement of every kernel of this library: with programmatic dependent
// launch (launch_kernel), a kernel may start while the one before it on the stream
// is finishing; this waits until that kernel has completed and its writes are
// visible, before any read or write of memory. A no-op for a normal launch.
// It then lets the next kernel on the stream launch (launch_dependents): that
// kernel's blocks may become resident while this one runs, and they wait in
// their own grid_dependency_wait until this whole grid has completed and its
// writes are visible, so an early trigger changes when blocks are placed, never
// what they read. BM_PDL_TRIGGER=0 at build time leaves the trigger to grid exit.
#ifndef BM_PDL_TRIGGER
#define BM_PDL_TRIGGER 1
#endif
#ifndef BM_PDL_PREFETCH
#define BM_PDL_PREFETCH 1
#endif

// Asks L2 for the 128-byte line holding p and does not wait for it. Kernels
// issue it for their first addresses before grid_dependency_wait, so the DRAM
// latency of their first loads overlaps the previous kernel instead of following
// it. It cannot change what a later load returns: L2 is where every SM's writes
// land, so a line fetched early and then written by the previous kernel holds
// the written bytes when this kernel reads it after the wait.
__device__ __forceinline__ void prefetch_l2(const void* p) {
#if BM_PDL_PREFETCH
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
#else
  (void)p;
#endif
}
// prefetch_l2 over [p, p + bytes), one line per participant per step.
__device__ __forceinline__ void prefetch_l2_range(const void* p, int64_t bytes, int idx, int count) {
  const char* c = static_cast<const char*>(p);
  for (int64_t off = static_cast<int64_t>(idx) * 128; off < bytes; off += static_cast<int64_t>(count) * 128) {
    prefetch_l2(c + off);
  }
}
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
#if BM_PDL_TRIGGER
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#endif
}

}  // namespace bm
