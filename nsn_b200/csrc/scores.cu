// Batched GQA decode scores over a per-channel quantised K cache (the K1c layout,
// experiments/kernels/phase_k1c_triton_fused_kernel.py:172-250):
//   codes u8 [B][T][n_kv*D] (one byte per value), min / step fp16 [B][n_kv*D] (per
//   channel over all T tokens), eff_norm fp16 [B][n_kv][T] (NSN only), q fp16 [B][n_q][D];
//   score[b][h][t] = (1/sqrt(D)) * eff_norm[b][h/rep][t] * sum_d q[b][h][d] * (code * step + min),
// with recipe FP16 reading K itself ([B][T][n_kv*D] fp16) and KIVI dropping eff_norm.
// One CTA takes 64 tokens of one (sequence, kv head) and serves all rep = n_q/n_kv
// query heads, so every code byte is read once (the reference's kernel runs one
// program per query head and reads the K tile rep times).
#include <cmath>

#include "nsnkv_common.cuh"

namespace nsnkv {

constexpr int kScTok = 64;        // tokens per CTA
constexpr int kScThreads = 128;   // thread (token, head parity)
constexpr int kScMaxDim = 256;
constexpr int kScMaxRep = 8;

template <bool FP16>
__global__ void __launch_bounds__(kScThreads) k1c_scores_kernel(int n_q, int n_kv, int64_t T, int D, int nsn,
                                                                 float inv_sqrt_d, const __half *q, const void *code,
                                                                 const uint16_t *kmin, const uint16_t *kstep,
                                                                 const uint16_t *enorm, float *out) {
  extern __shared__ __align__(16) unsigned char sm[];
  const int rep = n_q / n_kv;
  // shared: q [rep][D] fp32, min / step [D] fp32, then the K tile: 64 rows of D values
  // (bytes, or fp16 for FP16) with one extra 32-bit word per row so that the row reads
  // of consecutive threads fall in different banks.
  float *qs = reinterpret_cast<float *>(sm);
  float *mn = qs + rep * D, *st = mn + D;
  const int row_words = (FP16 ? D / 2 : D / 4) + 1;
  uint32_t *tile = reinterpret_cast<uint32_t *>(st + D);
  const int tid = threadIdx.x;
  const int64_t b = blockIdx.z, hk = blockIdx.y, t0 = static_cast<int64_t>(blockIdx.x) * kScTok;
  const int nt = static_cast<int>(T - t0 < kScTok ? T - t0 : kScTok);
  const int64_t hidden = static_cast<int64_t>(n_kv) * D;
  for (int e = tid; e < rep * D; e += kScThreads)
    qs[e] = __half2float(q[(b * n_q + hk * rep + e / D) * D + e % D]);
  if (!FP16) {
    for (int c = tid; c < D; c += kScThreads) {
      mn[c] = half_bits_to_f(kmin[b * hidden + hk * D + c]);
      st[c] = half_bits_to_f(kstep[b * hidden + hk * D + c]);
    }
  }
  // stage the tile with 16-byte loads (a token's D values of this head are contiguous)
  const int vec_per_row = FP16 ? D / 8 : D / 16;
  for (int e = tid; e < nt * vec_per_row; e += kScThreads) {
    const int t = e / vec_per_row, v = e % vec_per_row;
    const unsigned char *src = static_cast<const unsigned char *>(code) +
                               ((b * T + t0 + t) * hidden + hk * D) * (FP16 ? 2 : 1) + 16 * v;
    const uint4 x = *reinterpret_cast<const uint4 *>(src);
    uint32_t *dst = tile + t * row_words + 4 * v;
    dst[0] = x.x;
    dst[1] = x.y;
    dst[2] = x.z;
    dst[3] = x.w;
  }
  __syncthreads();
  const int t = tid & (kScTok - 1), par = tid >> 6;
  if (t >= nt) return;
  float acc[kScMaxRep / 2];
#pragma unroll
  for (int i = 0; i < kScMaxRep / 2; ++i) acc[i] = 0.f;
  const uint32_t *row = tile + t * row_words;
  if (FP16) {
    for (int w2 = 0; w2 < D / 2; ++w2) {
      const float2 k2 = Elem<__half>::to_f2(row[w2]);
#pragma unroll
      for (int i = 0; i < kScMaxRep / 2; ++i) {
        const int r = 2 * i + par;
        if (r < rep) acc[i] = fmaf(k2.y, qs[r * D + 2 * w2 + 1], fmaf(k2.x, qs[r * D + 2 * w2], acc[i]));
      }
    }
  } else {
    for (int w4 = 0; w4 < D / 4; ++w4) {
      const uint32_t word = row[w4];
      const float4 s4 = *reinterpret_cast<const float4 *>(&st[4 * w4]);
      const float4 m4 = *reinterpret_cast<const float4 *>(&mn[4 * w4]);
      const float sv[4] = {s4.x, s4.y, s4.z, s4.w}, mv[4] = {m4.x, m4.y, m4.z, m4.w};
      float kdq[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // the byte as the low mantissa of 2^23, minus 2^23: its exact float value
        const float code_f = __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7440 + j)) - 8388608.f;
        kdq[j] = fmaf(code_f, sv[j], mv[j]);
      }
#pragma unroll
      for (int i = 0; i < kScMaxRep / 2; ++i) {
        const int r = 2 * i + par;
        if (r < rep) {
          const float4 q4 = *reinterpret_cast<const float4 *>(&qs[r * D + 4 * w4]);
          acc[i] = fmaf(kdq[3], q4.w, fmaf(kdq[2], q4.z, fmaf(kdq[1], q4.y, fmaf(kdq[0], q4.x, acc[i]))));
        }
      }
    }
  }
  const float inv = inv_sqrt_d;
  const float en = nsn ? half_bits_to_f(enorm[(b * n_kv + hk) * T + t0 + t]) : 1.f;
#pragma unroll
  for (int i = 0; i < kScMaxRep / 2; ++i) {
    const int r = 2 * i + par;
    if (r < rep) out[(b * n_q + hk * rep + r) * T + t0 + t] = acc[i] * inv * en;
  }
}

}  // namespace nsnkv

using namespace nsnkv;

extern "C" int nsnkv_k1c_scores(int recipe, int64_t batch, int n_q, int n_kv, int64_t tokens, int head_dim,
                                const void *q, const void *code, const uint16_t *k_min, const uint16_t *k_step,
                                const uint16_t *eff_norm, float *scores, void *stream) {
  if (recipe < 0 || recipe > 2 || batch <= 0 || batch > 65535 || n_kv <= 0 || n_kv > 65535 || n_q <= 0 ||
      n_q % n_kv != 0 || n_q / n_kv > kScMaxRep || tokens <= 0 || head_dim < 16 || head_dim > kScMaxDim ||
      head_dim % 16 != 0)
    return NSNKV_ERR_ARG;
  if (!q || !code || !scores || (recipe != 0 && (!k_min || !k_step)) || (recipe == 2 && !eff_norm))
    return NSNKV_ERR_ARG;
  if (!aligned16(code)) return NSNKV_ERR_ARG;
  const bool fp16 = recipe == 0;
  const int rep = n_q / n_kv;
  const int row_words = (fp16 ? head_dim / 2 : head_dim / 4) + 1;
  const size_t smem = (static_cast<size_t>(rep) * head_dim + 2 * head_dim) * sizeof(float) +
                      static_cast<size_t>(kScTok) * row_words * sizeof(uint32_t);
  const dim3 grid(static_cast<unsigned>((tokens + kScTok - 1) / kScTok), static_cast<unsigned>(n_kv),
                  static_cast<unsigned>(batch));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto launch = [&](auto kernel) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return NSNKV_ERR_CUDA;
    kernel<<<grid, kScThreads, smem, st>>>(n_q, n_kv, tokens, head_dim, recipe == 2 ? 1 : 0,
                                           static_cast<float>(1.0 / std::sqrt(static_cast<double>(head_dim))),
                                           static_cast<const __half *>(q), code, k_min, k_step, eff_norm, scores);
    return cudaGetLastError() == cudaSuccess ? NSNKV_OK : NSNKV_ERR_LAUNCH;
  };
  return fp16 ? launch(k1c_scores_kernel<true>) : launch(k1c_scores_kernel<false>);
}
