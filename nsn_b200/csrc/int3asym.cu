// Int3AsymNsepPchanCache for sm_100a: the library's per-tensor INT3 container
// (src/nsn/cache.py:134-313).  A row of T tokens x D channels (D % 8 == 0, D <= 256)
// is stored as per-token fp16 norms, per-channel fp16 (d_min, d_step) of the unit
// directions over all T tokens, and 3-bit unsigned indices packed LSB first, 8 per 3
// bytes (src/nsn/pack.py:85-163).  Every operation reproduces the reference's CPU
// arithmetic bit for bit:
//   n = max(||x||, 1e-12) with the norm in torch's CPU order (8 lanes for a contiguous
//   row, sequential for a strided one), d = x / n,
//   d_min / d_max over tokens (a tie keeps the later token), step = max(d_max - d_min,
//   1e-12) / 7, idx = clamp(rint((d - d_min) / step), 0, 7);
//   decode: d_q = idx * step16 + min16, out = fp16(n16 * (d_q / max(||d_q||, 1e-8))).
#include "nsnkv_common.cuh"

namespace nsnkv {

constexpr int kAsymChunk = 64;   // tokens per CTA
constexpr int kAsymMaxDim = 256;
constexpr int kAsymThreads = 256;

// Sum of squares of a D-element row in torch's CPU order: lane j (0..7) accumulates
// x[j], x[j+8], ... (separately rounded multiply and add), then the lanes are added 0..7.
__device__ __forceinline__ float sumsq_lanes8_dim(const float *row, int D) {
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = mul_rn(row[j], row[j]);
  for (int i = 8; i < D; i += 8) {
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = add_rn(acc[j], mul_rn(row[i + j], row[i + j]));
  }
  float s = acc[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) s = add_rn(s, acc[j]);
  return s;
}

__device__ __forceinline__ float min_keep_later(float acc, float v) { return acc < v ? acc : v; }

// Pass 1: per-token clamped norms and, per 64-token chunk, each channel's min / max of d.
template <typename T>
__global__ void __launch_bounds__(kAsymThreads) asym_stats_kernel(const T *x, int64_t tokens, int D, int norm_order,
                                                                   int64_t nchunks, float *norms, float *pmin,
                                                                   float *pmax, int32_t *status) {
  extern __shared__ float xs[];  // [64][D + 1]
  __shared__ float tn[kAsymChunk];
  const int tid = threadIdx.x, ld = D + 1;
  const int64_t r = blockIdx.y, ch = blockIdx.x, c0 = ch * kAsymChunk;
  const int nt = static_cast<int>(tokens - c0 < kAsymChunk ? tokens - c0 : kAsymChunk);
  const T *src = x + (r * tokens + c0) * D;
  int bad = 0;
  for (int e = tid; e < nt * D; e += kAsymThreads) {
    const float f = Elem<T>::to_f(src[e]);
    bad |= !isfinite(f);
    xs[(e / D) * ld + e % D] = f;
  }
  __syncthreads();
  if (tid < nt) {
    const float *row = &xs[tid * ld];
    float ss;
    if (norm_order == 0) {
      ss = sumsq_lanes8_dim(row, D);
    } else {  // a strided row: torch sums sequentially
      ss = mul_rn(row[0], row[0]);
      for (int c = 1; c < D; ++c) ss = add_rn(ss, mul_rn(row[c], row[c]));
    }
    const float n = fmaxf(__fsqrt_rn(ss), 1e-12f);
    tn[tid] = n;
    norms[r * tokens + c0 + tid] = n;
  }
  __syncthreads();
  for (int e = tid; e < nt * D; e += kAsymThreads) {
    const int t = e / D, c = e % D;
    xs[t * ld + c] = div_rn(xs[t * ld + c], tn[t]);
  }
  __syncthreads();
  for (int c = tid; c < D; c += kAsymThreads) {
    float lo = xs[c], hi = xs[c];
    for (int t = 1; t < nt; ++t) {
      const float v = xs[t * ld + c];
      lo = min_keep_later(lo, v);
      hi = fmaxf(hi, v);
    }
    pmin[(r * nchunks + ch) * D + c] = lo;
    pmax[(r * nchunks + ch) * D + c] = hi;
  }
  if (bad) set_status(status, NSNKV_ST_INPUT_NONFINITE);
}

// Pass 2: chunk partials in token order -> d_min, d_step (fp32 for the codes, fp16 stored).
__global__ void __launch_bounds__(kAsymThreads) asym_meta_kernel(int64_t nchunks, int D, const float *pmin,
                                                                  const float *pmax, float *fmin, float *fstep,
                                                                  uint16_t *d_min, uint16_t *d_step) {
  const int64_t r = blockIdx.x;
  for (int c = threadIdx.x; c < D; c += kAsymThreads) {
    float lo = pmin[r * nchunks * D + c], hi = pmax[r * nchunks * D + c];
    for (int64_t k = 1; k < nchunks; ++k) {
      lo = min_keep_later(lo, pmin[(r * nchunks + k) * D + c]);
      hi = fmaxf(hi, pmax[(r * nchunks + k) * D + c]);
    }
    const float step = div_rn(fmaxf(sub_rn(hi, lo), 1e-12f), 7.f);
    fmin[r * D + c] = lo;
    fstep[r * D + c] = step;
    d_min[r * D + c] = f_to_half_bits(lo);
    d_step[r * D + c] = f_to_half_bits(step);
  }
}

// Pass 3: indices of 8 consecutive channels of one token -> 3 packed bytes; fp16 norms.
template <typename T>
__global__ void __launch_bounds__(kAsymThreads) asym_codes_kernel(const T *x, int64_t tokens, int D,
                                                                   const float *norms, const float *fmin,
                                                                   const float *fstep, uint8_t *packed,
                                                                   uint16_t *norm16) {
  const int64_t r = blockIdx.y, c0 = static_cast<int64_t>(blockIdx.x) * kAsymChunk;
  const int nt = static_cast<int>(tokens - c0 < kAsymChunk ? tokens - c0 : kAsymChunk);
  const int groups = D / 8;
  for (int e = threadIdx.x; e < nt * groups; e += kAsymThreads) {
    const int t = e / groups, gidx = e % groups;
    const int64_t tok = r * tokens + c0 + t;
    const float n = norms[tok];
    uint32_t v = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = 8 * gidx + j;
      const float d = div_rn(Elem<T>::to_f(x[tok * D + c]), n);
      float q = rintf(div_rn(sub_rn(d, fmin[r * D + c]), fstep[r * D + c]));
      q = fminf(fmaxf(q, 0.f), 7.f);
      v |= static_cast<uint32_t>(q) << (3 * j);
    }
    uint8_t *dst = packed + tok * (3 * D / 8) + 3 * gidx;
    dst[0] = static_cast<uint8_t>(v);
    dst[1] = static_cast<uint8_t>(v >> 8);
    dst[2] = static_cast<uint8_t>(v >> 16);
    if (gidx == 0) norm16[tok] = f_to_half_bits(n);
  }
}

// Decode: d_q = idx * step16 + min16, renormalised, times the fp16 norm, rounded to fp16.
__global__ void __launch_bounds__(kAsymThreads) asym_decode_kernel(const uint8_t *packed, const uint16_t *norm16,
                                                                    const uint16_t *d_min, const uint16_t *d_step,
                                                                    int64_t tokens, int D, uint16_t *out) {
  extern __shared__ float dq[];  // [64][D + 1]
  __shared__ float scale[kAsymChunk];
  const int tid = threadIdx.x, ld = D + 1, groups = D / 8;
  const int64_t r = blockIdx.y, c0 = static_cast<int64_t>(blockIdx.x) * kAsymChunk;
  const int nt = static_cast<int>(tokens - c0 < kAsymChunk ? tokens - c0 : kAsymChunk);
  for (int e = tid; e < nt * groups; e += kAsymThreads) {
    const int t = e / groups, gidx = e % groups;
    const uint8_t *src = packed + (r * tokens + c0 + t) * (3 * D / 8) + 3 * gidx;
    const uint32_t v = src[0] | (static_cast<uint32_t>(src[1]) << 8) | (static_cast<uint32_t>(src[2]) << 16);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = 8 * gidx + j;
      const float idx = static_cast<float>((v >> (3 * j)) & 7u);
      dq[t * ld + c] = add_rn(mul_rn(idx, half_bits_to_f(d_step[r * D + c])), half_bits_to_f(d_min[r * D + c]));
    }
  }
  __syncthreads();
  if (tid < nt) scale[tid] = fmaxf(__fsqrt_rn(sumsq_lanes8_dim(&dq[tid * ld], D)), 1e-8f);
  __syncthreads();
  for (int e = tid; e < nt * D; e += kAsymThreads) {
    const int t = e / D, c = e % D;
    const float n = half_bits_to_f(norm16[r * tokens + c0 + t]);
    out[(r * tokens + c0 + t) * D + c] = f_to_half_bits(mul_rn(n, div_rn(dq[t * ld + c], scale[t])));
  }
}

static bool asym_shape_ok(int64_t rows, int64_t tokens, int dim) {
  return rows > 0 && rows <= 65535 && tokens > 0 && dim >= 8 && dim <= kAsymMaxDim && dim % 8 == 0 &&
         (tokens + kAsymChunk - 1) / kAsymChunk <= 0x7FFFFFFF;
}

static int64_t asym_scratch_floats(int64_t rows, int64_t tokens, int dim) {
  const int64_t nchunks = (tokens + kAsymChunk - 1) / kAsymChunk;
  return rows * tokens + 2 * rows * nchunks * dim + 2 * rows * dim;
}

template <typename T>
static int asym_encode(const void *x, int64_t rows, int64_t tokens, int dim, int norm_order, uint8_t *packed,
                       uint16_t *norm, uint16_t *d_min, uint16_t *d_step, float *scratch, int32_t *status,
                       cudaStream_t st) {
  const int64_t nchunks = (tokens + kAsymChunk - 1) / kAsymChunk;
  float *norms = scratch, *pmin = norms + rows * tokens, *pmax = pmin + rows * nchunks * dim;
  float *fmin = pmax + rows * nchunks * dim, *fstep = fmin + rows * dim;
  const size_t smem = static_cast<size_t>(kAsymChunk) * (dim + 1) * sizeof(float);
  auto k1 = asym_stats_kernel<T>;
  if (cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return NSNKV_ERR_CUDA;
  const dim3 grid(static_cast<unsigned>(nchunks), static_cast<unsigned>(rows));
  k1<<<grid, kAsymThreads, smem, st>>>(static_cast<const T *>(x), tokens, dim, norm_order, nchunks, norms, pmin,
                                       pmax, status);
  asym_meta_kernel<<<static_cast<unsigned>(rows), kAsymThreads, 0, st>>>(nchunks, dim, pmin, pmax, fmin, fstep, d_min,
                                                                         d_step);
  asym_codes_kernel<T><<<grid, kAsymThreads, 0, st>>>(static_cast<const T *>(x), tokens, dim, norms, fmin, fstep,
                                                      packed, norm);
  return cudaGetLastError() == cudaSuccess ? NSNKV_OK : NSNKV_ERR_LAUNCH;
}

}  // namespace nsnkv

using namespace nsnkv;

extern "C" {

int64_t nsnkv_int3asym_scratch_bytes(int64_t rows, int64_t tokens, int dim) {
  if (!asym_shape_ok(rows, tokens, dim)) return 0;
  return asym_scratch_floats(rows, tokens, dim) * static_cast<int64_t>(sizeof(float));
}

int nsnkv_int3asym_encode(const void *x, int x_dtype, int64_t rows, int64_t tokens, int dim, int norm_order,
                          uint8_t *packed, uint16_t *norm, uint16_t *d_min, uint16_t *d_step, void *scratch,
                          int64_t scratch_bytes, int32_t *status, void *stream) {
  if (!asym_shape_ok(rows, tokens, dim) || !x || !packed || !norm || !d_min || !d_step || !scratch || !status)
    return NSNKV_ERR_ARG;
  if (norm_order != 0 && norm_order != 1) return NSNKV_ERR_ARG;
  if (scratch_bytes < nsnkv_int3asym_scratch_bytes(rows, tokens, dim)) return NSNKV_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float *s = static_cast<float *>(scratch);
  switch (x_dtype) {
    case NSNKV_F16:
      return asym_encode<__half>(x, rows, tokens, dim, norm_order, packed, norm, d_min, d_step, s, status, st);
    case NSNKV_BF16:
      return asym_encode<__nv_bfloat16>(x, rows, tokens, dim, norm_order, packed, norm, d_min, d_step, s, status, st);
    case NSNKV_F32:
      return asym_encode<float>(x, rows, tokens, dim, norm_order, packed, norm, d_min, d_step, s, status, st);
    default: return NSNKV_ERR_ARG;
  }
}

int nsnkv_int3asym_decode(const uint8_t *packed, const uint16_t *norm, const uint16_t *d_min, const uint16_t *d_step,
                          int64_t rows, int64_t tokens, int dim, uint16_t *out, void *stream) {
  if (!asym_shape_ok(rows, tokens, dim) || !packed || !norm || !d_min || !d_step || !out) return NSNKV_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t smem = static_cast<size_t>(kAsymChunk) * (dim + 1) * sizeof(float);
  if (cudaFuncSetAttribute(asym_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return NSNKV_ERR_CUDA;
  const int64_t nchunks = (tokens + kAsymChunk - 1) / kAsymChunk;
  asym_decode_kernel<<<dim3(static_cast<unsigned>(nchunks), static_cast<unsigned>(rows)), kAsymThreads, smem, st>>>(
      packed, norm, d_min, d_step, tokens, dim, out);
  return cudaGetLastError() == cudaSuccess ? NSNKV_OK : NSNKV_ERR_LAUNCH;
}

}  // extern "C"
