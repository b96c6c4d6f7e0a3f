// Split-KV record exchange over peer memory, fused with the log-sum-exp merge.
//
// After each rank's local attention over its block range, the ranks' (o, lse) records
// must meet (the reference merges chunk partials on one GPU,
// experiments/ac08/source/loop_kv_af01_kernel.py:70-84; across GPUs the records
// travel first).  Instead of an NCCL all-gather followed by a merge kernel, one kernel
// per rank writes its record straight into every peer's memory over NVLink (plain P2P
// stores into a symmetric area every rank maps) and merges as soon as the peers' records
// have landed in its own area.
//
// Area (the same layout on every rank, fp32 words):
//   recv [2][world][hq * 129]   parity e & 1 of the call, slot s = rank s's record:
//                               o [hq][128] then lse [hq]
//   flags [world][hq] (uint32)  flag (s, h) = the epoch of rank s's latest push of head h
// One CTA of 128 threads per query head h:
//   1. push: rank r's o row h and lse h into slot r of every peer's recv, then, after a
//      system-scope fence, flag (r, h) = e in every peer (release store);
//   2. wait: thread 0 polls its own flags (s, h) until every rank reached e (acquire loads;
//      bounded: NSNKV_ST_TIMEOUT and no output when a peer never arrives);
//   3. merge in rank order, the arithmetic of merge_shards_kernel.
// epochs[h] (this rank's device memory) counts the calls, so a replayed CUDA graph moves
// on to the next epoch.  A rank is at most one call ahead of another (its next push needs
// every peer's current one), so two parities keep a record from being overwritten before
// it is merged, and flags compare as "at least e".
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "nsnkv_common.cuh"

namespace nsnkv {
namespace {

constexpr uint32_t kPeerPolls = 1u << 22;  // about a second with the back-off below

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <typename T>
__global__ void __launch_bounds__(128) peer_merge_kernel(int world, int rank, int hq, const float *rec,
                                                         float *const *peers, float *area, uint32_t *epochs, T *out,
                                                         float *out_f32, float *lse_out, int32_t *status) {
  const int h = blockIdx.x, c = threadIdx.x;
  const int64_t slot = static_cast<int64_t>(hq) * (kDim + 1);
  const uint32_t e = epochs[h] + 1u;
  const int64_t par = static_cast<int64_t>(e & 1u) * world * slot;
  const float ov = rec[static_cast<int64_t>(h) * kDim + c];
  const float lv = rec[static_cast<int64_t>(hq) * kDim + h];
  for (int s = 0; s < world; ++s) {
    float *dst = peers[s] + par + rank * slot;
    dst[static_cast<int64_t>(h) * kDim + c] = ov;
    if (c == 0) dst[static_cast<int64_t>(hq) * kDim + h] = lv;
  }
  __threadfence_system();
  __syncthreads();  // every thread's stores are ordered before thread 0's flags
  __shared__ int arrived;
  if (c == 0) {
    for (int s = 0; s < world; ++s)
      st_release_sys(reinterpret_cast<uint32_t *>(peers[s] + 2 * world * slot) + rank * hq + h, e);
    const uint32_t *flags = reinterpret_cast<const uint32_t *>(area + 2 * world * slot);
    int all = 0;
    for (uint32_t it = 0; it < kPeerPolls && !all; ++it) {
      all = 1;
      for (int s = 0; s < world && all; ++s)
        all = static_cast<int32_t>(ld_acquire_sys(flags + s * hq + h) - e) >= 0;
      if (!all && it > 64) __nanosleep(128);
    }
    arrived = all;
    if (!all) set_status(status, NSNKV_ST_TIMEOUT);
    epochs[h] = e;
  }
  __syncthreads();
  if (!arrived) return;
  const float *recv = area + par;
  float M = -INFINITY;
  for (int s = 0; s < world; ++s) M = fmaxf(M, __ldcg(recv + s * slot + static_cast<int64_t>(hq) * kDim + h));
  float L = 0.f, acc = 0.f;
  for (int s = 0; s < world; ++s) {
    const float l = __ldcg(recv + s * slot + static_cast<int64_t>(hq) * kDim + h);
    const float w = l == -INFINITY ? 0.f : expf(l - M);
    L += w;
    acc += w * __ldcg(recv + s * slot + static_cast<int64_t>(h) * kDim + c);
  }
  const float y = __fdiv_rn(acc, L);
  const T yt = Elem<T>::from_f(y);
  out[static_cast<int64_t>(h) * kDim + c] = yt;
  if (out_f32) out_f32[static_cast<int64_t>(h) * kDim + c] = y;
  if (lse_out && c == 0) lse_out[h] = M + logf(L);
  if (!isfinite(Elem<T>::to_f(yt))) set_status(status, NSNKV_ST_OUTPUT_NONFINITE);
}

}  // namespace
}  // namespace nsnkv

using namespace nsnkv;

extern "C" {

int64_t nsnkv_peer_area_words(int world, int hq) {
  if (world <= 0 || hq <= 0) return 0;
  return 2LL * world * hq * (kDim + 1) + static_cast<int64_t>(world) * hq;
}

int nsnkv_peer_merge_records(int world, int rank, int hq, int dtype, const float *record, void *const *peer_areas,
                             float *area, uint32_t *epochs, void *out, float *out_f32, float *lse_out,
                             int32_t *status, void *stream) {
  if (world <= 0 || rank < 0 || rank >= world || hq <= 0 || hq > 65535) return NSNKV_ERR_ARG;
  if (dtype != NSNKV_F16 && dtype != NSNKV_BF16) return NSNKV_ERR_ARG;
  if (!record || !peer_areas || !area || !epochs || !out || !status) return NSNKV_ERR_ARG;
  if (!aligned16(area)) return NSNKV_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float *const *peers = reinterpret_cast<float *const *>(peer_areas);
  if (dtype == NSNKV_F16)
    peer_merge_kernel<__half><<<hq, kDim, 0, st>>>(world, rank, hq, record, peers, area, epochs,
                                                   static_cast<__half *>(out), out_f32, lse_out, status);
  else
    peer_merge_kernel<__nv_bfloat16><<<hq, kDim, 0, st>>>(world, rank, hq, record, peers, area, epochs,
                                                          static_cast<__nv_bfloat16 *>(out), out_f32, lse_out,
                                                          status);
  return cudaGetLastError() == cudaSuccess ? NSNKV_OK : NSNKV_ERR_LAUNCH;
}

}  // extern "C"
