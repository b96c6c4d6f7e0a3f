// Shared device helpers for the NSN packed-KV kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/nsnkv.h"

namespace nsnkv {

constexpr int kBlock = 64;   // tokens per sealed block
constexpr int kDim = 128;    // head_dim
constexpr float kEps = 1e-12f;
constexpr float kScale = 0.08838834764831845f;  // 1/sqrt(128)

__host__ __device__ constexpr int code_bytes(int bits) { return kBlock * kDim * bits / 8; }
// Byte b of token t's packed code row inside a block, for the block's code order:
//   0  the reference's rows back to back (LSB-first bitstream);
//   1  paired rows (the V codes of the paged cache's block records): the rows of tokens 2j
//      and 2j+1 interleaved at 16 bits, 32-bit word j*8*bits + k = [row 2j half k | row 2j+1 half k];
//   2  paired halves (the K codes of the block records): in each row, each 32-code group
//      (2*bits 16-bit halves, A = the first bits halves, B = the rest) stored as words
//      [A half m | B half m], m < bits.
__host__ __device__ __forceinline__ int code_byte_at(int t, int b, int bits, int order) {
  if (order == 1) return 4 * ((t >> 1) * 8 * bits + (b >> 1)) + 2 * (t & 1) + (b & 1);
  if (order == 2) {
    const int gb = b % (4 * bits), hh = gb >> 1;
    const int out_half = hh < bits ? 2 * hh : 2 * (hh - bits) + 1;
    return t * 16 * bits + (b - gb) + 2 * out_half + (gb & 1);
  }
  return t * 16 * bits + b;
}

// Block i of an array whose blocks are `bytes` apart (a dense array, or one field of the
// paged cache's block records).
template <typename T>
__host__ __device__ __forceinline__ T *blk_ptr(T *base, int64_t i, int64_t bytes) {
  return reinterpret_cast<T *>(reinterpret_cast<uintptr_t>(base) + static_cast<uintptr_t>(i * bytes));
}

// ----------------------------------------------------------------- dtype helpers
template <typename T> struct Elem;
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float2 to_f2(uint32_t bits) {
    __half2 h = *reinterpret_cast<__half2 *>(&bits);
    return __half22float2(h);
  }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float2 to_f2(uint32_t bits) {
    return make_float2(__uint_as_float(bits << 16), __uint_as_float(bits & 0xFFFF0000u));
  }
};
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};

__device__ __forceinline__ float half_bits_to_f(uint16_t b) { return __half2float(__ushort_as_half(b)); }
__device__ __forceinline__ uint16_t f_to_half_bits(float v) { return __half_as_ushort(__float2half_rn(v)); }

__device__ __forceinline__ bool finite_f(float v) { return isfinite(v); }

__device__ __forceinline__ void set_status(int32_t *status, int bits) {
  if (bits && status) atomicOr(status, bits);
}

// ----------------------------------------------------------------- exact float ops
// The reference's CPU arithmetic rounds every multiply and add separately; these
// wrappers keep the compiler from contracting them into fused multiply-adds.
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float div_rn(float a, float b) { return __fdiv_rn(a, b); }

// Sum of squares of one 128-element row in torch's CPU order for a contiguous row:
// lane j (0..7) accumulates x[j], x[j+8], ..., x[j+120]; lanes are then added 0..7.
// `row` points at the row; `stride` is the element stride (1 for a packed row).
__device__ __forceinline__ float sumsq_lanes8(const float *row, int stride) {
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = mul_rn(row[j * stride], row[j * stride]);
#pragma unroll
  for (int i = 8; i < kDim; i += 8) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float v = row[(i + j) * stride];
      acc[j] = add_rn(acc[j], mul_rn(v, v));
    }
  }
  float s = acc[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) s = add_rn(s, acc[j]);
  return s;
}

// Plain sequential sum of squares (torch's order for a row with strided channels).
__device__ __forceinline__ float sumsq_seq(const float *row, int stride) {
  float s = mul_rn(row[0], row[0]);
#pragma unroll 8
  for (int c = 1; c < kDim; ++c) {
    float v = row[c * stride];
    s = add_rn(s, mul_rn(v, v));
  }
  return s;
}

// ----------------------------------------------------------------- bounded mbarrier waits
// Every wait below gives up after a fixed number of polls, sets
// NSNKV_ST_TIMEOUT and reports failure so the kernel can return.
constexpr uint32_t kWaitPolls = 1u << 22;

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t phase) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(a), "r"(phase)
      : "memory");
  return ok != 0;
}

// Returns false (after setting the timeout status) when the phase never completes.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t phase, int32_t *status) {
  for (uint32_t i = 0; i < kWaitPolls; ++i) {
    if (mbar_try_wait(bar, phase)) return true;
    if (i > 64) __nanosleep(64);
  }
  set_status(status, NSNKV_ST_TIMEOUT);
  return false;
}

// 1-D bulk copy global -> shared (TMA engine), completion counted on `bar`.
// dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  uint32_t b = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(d),
      "l"(src), "r"(bytes), "r"(b)
      : "memory");
}

// d += A * B, m16n8k16, A row-major and B column-major fragments of T (fp16 or bf16), fp32 d.
template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                 uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace nsnkv
