// Fused per-token layer ops of the looped decoder's decode step (nsn_b200/looped.py).
//
// At decode the model's rows are few (one token per sequence), so each torch elementwise op
// is its own small launch: the RMSNorm alone is six (upcast, square, mean, rsqrt, scale,
// weight), RoPE about eight.  These kernels do each group in one launch, in the rounding
// order of the transformers Llama modules the reference's adapter patches
// (experiments/ac08/source/loop_kv_ac08_attention.py:46-96 calls them):
//   add_rmsnorm  h = x + r (rounded to the dtype); y = w * dtype(h32 * rsqrt(mean(h32^2) + eps))
//                (LlamaRMSNorm: fp32 statistics, the normalised row cast back, then the weight)
//   rope_split   q = dtype(q * cos) + dtype(rotate_half(q) * sin), the same for k, v copied,
//                from one fused q|k|v projection row into the contiguous q, k, v the paged
//                cache step takes (apply_rotary_pos_emb)
//   swiglu       y = dtype(silu(g)) * u from one fused gate|up projection row (LlamaMLP's
//                act_fn(gate_proj(x)) * up_proj(x), silu computed in fp32)
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "nsnkv_common.cuh"

namespace nsnkv {
namespace {

template <typename T> __device__ __forceinline__ float tf(T x);
template <> __device__ __forceinline__ float tf<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float tf<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> __device__ __forceinline__ T ft(float x);
template <> __device__ __forceinline__ __half ft<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 ft<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

constexpr int kNormThreads = 256;

// Programmatic dependent launch.  Every kernel here is launched with programmatic stream
// serialisation, so it may become resident while the kernel before it on the stream is
// still running.  It waits (griddepcontrol.wait: that kernel complete and its writes
// visible) before it reads anything that kernel may have written, and only after the wait
// lets the kernel after it launch.  So a kernel that starts early never overlaps any
// kernel but its immediate predecessor, which has itself passed its own wait.
__device__ __forceinline__ void dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void dep_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
int launch_dep(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...) == cudaSuccess ? NSNKV_OK : NSNKV_ERR_LAUNCH;
}

// One CTA per row.  Each thread keeps its elements in registers between the two passes.
template <typename T, int PER>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(const T *x, const T *r, const T *w, float eps,
                                                                    int dim, T *res_out, T *y) {
  dep_wait();
  dep_release();
  const int64_t row = blockIdx.x;
  const T *xr = x + row * dim;
  const T *rr = r ? r + row * dim : nullptr;
  float hv[PER];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = threadIdx.x + i * kNormThreads;
    float v = 0.f;
    if (c < dim) {
      T hs = xr[c];
      if (rr) hs = ft<T>(tf<T>(hs) + tf<T>(rr[c]));  // the residual add, rounded to the dtype
      if (res_out) res_out[row * dim + c] = hs;
      v = tf<T>(hs);
    }
    hv[i] = v;
    ss = fmaf(v, v, ss);
  }
  __shared__ float red[kNormThreads / 32];
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float rs = rsqrtf(tot / static_cast<float>(dim) + eps);
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = threadIdx.x + i * kNormThreads;
    if (c < dim) y[row * dim + c] = ft<T>(tf<T>(w[c]) * tf<T>(ft<T>(hv[i] * rs)));
  }
}

// One CTA of 64 threads per (row, head): thread i rotates the pair (i, i + 64) of a 128-wide head.
template <typename T>
__global__ void __launch_bounds__(64) rope_split_kernel(const T *qkv, const T *cs, const T *sn, int64_t cs_stride,
                                                        int hq, int h, T *q, T *k, T *v) {
  dep_wait();
  dep_release();
  const int64_t row = blockIdx.y;
  const int head = blockIdx.x;  // 0 .. hq + 2h - 1 over the fused row's q, k, v heads
  const int i = threadIdx.x;
  const int width = (hq + 2 * h) * kDim;
  const T *src = qkv + row * width + static_cast<int64_t>(head) * kDim;
  if (head >= hq + h) {  // v: a copy
    T *dst = v + (row * h + (head - hq - h)) * kDim;
    dst[i] = src[i];
    dst[i + 64] = src[i + 64];
    return;
  }
  T *dst = head < hq ? q + (row * hq + head) * kDim : k + (row * h + (head - hq)) * kDim;
  const T *c = cs + row * cs_stride, *s = sn + row * cs_stride;
  const float x0 = tf<T>(src[i]), x1 = tf<T>(src[i + 64]);
  // rotate_half: [-x1, x0]
  dst[i] = ft<T>(tf<T>(ft<T>(x0 * tf<T>(c[i]))) + tf<T>(ft<T>(-x1 * tf<T>(s[i]))));
  dst[i + 64] = ft<T>(tf<T>(ft<T>(x1 * tf<T>(c[i + 64]))) + tf<T>(ft<T>(x0 * tf<T>(s[i + 64]))));
}

template <typename T>
__global__ void swiglu_kernel(const T *gu, int64_t rows, int inter, T *y) {
  dep_wait();
  dep_release();
  const int64_t n = rows * inter;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = e / inter, c = e % inter;
    const float g = tf<T>(gu[row * 2 * inter + c]);
    const float u = tf<T>(gu[row * 2 * inter + inter + c]);
    const float act = g / (1.f + expf(-g));
    y[e] = ft<T>(tf<T>(ft<T>(act)) * u);
  }
}

// Y [m][n] = X [m][k] . W [n][k]^T for the few rows of a decode step (m <= 8): the weight
// rows stream from HBM once, 16 bytes per lane, into mma.sync with fp32 accumulation.  A
// CTA of 8 warps owns 8 output columns (8 weight rows); warp w takes the k range
// [w k/8, (w+1) k/8).  Lane (g, t) loads 16 contiguous bytes of weight row n0 + g at
// k0 + 8t and the same k of X row g; the k order inside each 32-wide block is permuted
// alike for A and B (MMA slot 2t+j of k-step 0 <- k0 + 8t + j, slot 2t+8+j <- k0 + 8t + 2 + j;
// k-step 1 takes k0 + 8t + 4..7), which leaves the dot products unchanged.  X rows past
// m are zero; the warps' fp32 partials meet in shared memory.  With fixed_w (weights that
// no work still running on the stream writes: model weights while decoding) a lane's first
// weight vectors are loaded before the programmatic wait, so the weight stream starts
// while the kernel before this one finishes; x is read only after the wait.
template <typename T>
__global__ void __launch_bounds__(256) gemv_rows_kernel(const T *x, const T *w, T *y, int m, int n, int k,
                                                        int fixed_w) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int n0 = blockIdx.x * 8;
  const int span = k / 8;
  const int kb0 = warp * span + 8 * t;
  const uint4 *wp = reinterpret_cast<const uint4 *>(w + static_cast<int64_t>(n0 + g) * k + kb0);
  const uint4 *xp = reinterpret_cast<const uint4 *>(x + static_cast<int64_t>(g) * k + kb0);
  const bool row = g < m;
  float c[4] = {0.f, 0.f, 0.f, 0.f};
  constexpr int kUnroll = 4;
  int it = 0;
  const int iters = span / 32;  // 32-wide k blocks of this warp: one uint4 (8 of the block's 32 k) per lane
  if (fixed_w && iters >= kUnroll) {
    uint4 wv[kUnroll], xv[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) wv[u] = __ldcs(wp + 4 * u);
    dep_wait();
    dep_release();
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) xv[u] = row ? xp[4 * u] : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      mma16816<T>(c, xv[u].x, 0u, xv[u].y, 0u, wv[u].x, wv[u].y);
      mma16816<T>(c, xv[u].z, 0u, xv[u].w, 0u, wv[u].z, wv[u].w);
    }
    it = kUnroll;
  } else {
    dep_wait();
    dep_release();
  }
  for (; it + kUnroll <= iters; it += kUnroll) {
    uint4 wv[kUnroll], xv[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      wv[u] = __ldcs(wp + 4 * (it + u));
      xv[u] = row ? xp[4 * (it + u)] : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      mma16816<T>(c, xv[u].x, 0u, xv[u].y, 0u, wv[u].x, wv[u].y);
      mma16816<T>(c, xv[u].z, 0u, xv[u].w, 0u, wv[u].z, wv[u].w);
    }
  }
  for (; it < iters; ++it) {
    const uint4 wv = __ldcs(wp + 4 * it);
    const uint4 xv = row ? xp[4 * it] : make_uint4(0u, 0u, 0u, 0u);
    mma16816<T>(c, xv.x, 0u, xv.y, 0u, wv.x, wv.y);
    mma16816<T>(c, xv.z, 0u, xv.w, 0u, wv.z, wv.w);
  }
  __shared__ float part[8][8][8];  // [warp][row][column]
  part[warp][g][2 * t] = c[0];
  part[warp][g][2 * t + 1] = c[1];
  __syncthreads();
  if (threadIdx.x < 64) {
    const int r = threadIdx.x >> 3, col = threadIdx.x & 7;
    if (r < m) {
      float s = 0.f;
#pragma unroll
      for (int wi = 0; wi < 8; ++wi) s += part[wi][r][col];
      y[static_cast<int64_t>(r) * n + n0 + col] = ft<T>(s);
    }
  }
}

template <typename T>
int add_rmsnorm_launch(int64_t rows, int dim, const void *x, const void *r, const void *w, float eps, void *res_out,
                       void *y, cudaStream_t st) {
  const T *xp = static_cast<const T *>(x), *rp = static_cast<const T *>(r), *wp = static_cast<const T *>(w);
  T *ro = static_cast<T *>(res_out), *yp = static_cast<T *>(y);
  const dim3 grid(static_cast<unsigned>(rows));
  const dim3 block(kNormThreads);
  if (dim <= 4 * kNormThreads) return launch_dep(add_rmsnorm_kernel<T, 4>, grid, block, st, xp, rp, wp, eps, dim, ro, yp);
  if (dim <= 8 * kNormThreads) return launch_dep(add_rmsnorm_kernel<T, 8>, grid, block, st, xp, rp, wp, eps, dim, ro, yp);
  return launch_dep(add_rmsnorm_kernel<T, 32>, grid, block, st, xp, rp, wp, eps, dim, ro, yp);
}

}  // namespace
}  // namespace nsnkv

using namespace nsnkv;

extern "C" {

int nsnkv_add_rmsnorm(int64_t rows, int dim, int dtype, const void *x, const void *residual, const void *weight,
                      float eps, void *residual_out, void *out, void *stream) {
  if (rows < 0 || dim <= 0 || dim > 32 * kNormThreads || !(eps >= 0.f)) return NSNKV_ERR_ARG;
  if (dtype != NSNKV_F16 && dtype != NSNKV_BF16) return NSNKV_ERR_ARG;
  if (rows == 0) return NSNKV_OK;
  if (!x || !weight || !out || rows > 0x7fffffffLL) return NSNKV_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == NSNKV_F16 ? add_rmsnorm_launch<__half>(rows, dim, x, residual, weight, eps, residual_out, out, st)
                            : add_rmsnorm_launch<__nv_bfloat16>(rows, dim, x, residual, weight, eps, residual_out,
                                                                out, st);
}

int nsnkv_rope_split(int64_t rows, int hq, int h, int dtype, const void *qkv, const void *cos, const void *sin,
                     int64_t cs_stride, void *q, void *k, void *v, void *stream) {
  if (rows < 0 || hq <= 0 || h <= 0 || cs_stride < 0) return NSNKV_ERR_ARG;
  if (dtype != NSNKV_F16 && dtype != NSNKV_BF16) return NSNKV_ERR_ARG;
  if (rows == 0) return NSNKV_OK;
  if (!qkv || !cos || !sin || !q || !k || !v || rows > 65535 || hq + 2 * h > 65535) return NSNKV_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>(hq + 2 * h), static_cast<unsigned>(rows));
  if (dtype == NSNKV_F16)
    return launch_dep(rope_split_kernel<__half>, grid, dim3(64), st, static_cast<const __half *>(qkv),
                      static_cast<const __half *>(cos), static_cast<const __half *>(sin), cs_stride, hq, h,
                      static_cast<__half *>(q), static_cast<__half *>(k), static_cast<__half *>(v));
  return launch_dep(rope_split_kernel<__nv_bfloat16>, grid, dim3(64), st, static_cast<const __nv_bfloat16 *>(qkv),
                    static_cast<const __nv_bfloat16 *>(cos), static_cast<const __nv_bfloat16 *>(sin), cs_stride, hq,
                    h, static_cast<__nv_bfloat16 *>(q), static_cast<__nv_bfloat16 *>(k),
                    static_cast<__nv_bfloat16 *>(v));
}

int nsnkv_gemv_rows(int m, int n, int k, int dtype, const void *x, const void *w, void *y, int flags, void *stream) {
  if (m < 0 || m > 8 || n < 0 || k < 0 || n % 8 != 0 || k % 256 != 0) return NSNKV_ERR_ARG;
  if (dtype != NSNKV_F16 && dtype != NSNKV_BF16) return NSNKV_ERR_ARG;
  if (flags & ~NSNKV_GEMV_FIXED_WEIGHTS) return NSNKV_ERR_ARG;
  if (m == 0 || n == 0) return NSNKV_OK;
  if (!x || !w || !y || !aligned16(x) || !aligned16(w) || k == 0 || n / 8 > 0x7fffffff) return NSNKV_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>(n / 8));
  const int fixed_w = (flags & NSNKV_GEMV_FIXED_WEIGHTS) ? 1 : 0;
  if (dtype == NSNKV_F16)
    return launch_dep(gemv_rows_kernel<__half>, grid, dim3(256), st, static_cast<const __half *>(x),
                      static_cast<const __half *>(w), static_cast<__half *>(y), m, n, k, fixed_w);
  return launch_dep(gemv_rows_kernel<__nv_bfloat16>, grid, dim3(256), st, static_cast<const __nv_bfloat16 *>(x),
                    static_cast<const __nv_bfloat16 *>(w), static_cast<__nv_bfloat16 *>(y), m, n, k, fixed_w);
}

int nsnkv_swiglu(int64_t rows, int inter, int dtype, const void *gate_up, void *out, void *stream) {
  if (rows < 0 || inter <= 0) return NSNKV_ERR_ARG;
  if (dtype != NSNKV_F16 && dtype != NSNKV_BF16) return NSNKV_ERR_ARG;
  if (rows == 0) return NSNKV_OK;
  if (!gate_up || !out) return NSNKV_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t n = rows * inter;
  const unsigned blocks = static_cast<unsigned>(n / 256 + 1 < 148 * 8 ? n / 256 + 1 : 148 * 8);
  if (dtype == NSNKV_F16)
    return launch_dep(swiglu_kernel<__half>, dim3(blocks), dim3(256), st, static_cast<const __half *>(gate_up), rows,
                      inter, static_cast<__half *>(out));
  return launch_dep(swiglu_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), st,
                    static_cast<const __nv_bfloat16 *>(gate_up), rows, inter, static_cast<__nv_bfloat16 *>(out));
}

}  // extern "C"
