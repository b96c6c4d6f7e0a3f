// Decode-step plans over a paged packed-KV cache (include/nsnkv.h, nsnkv_paged_*).
//
// A batched decode step is one attention launch chain (nsnkv_decode_attn_alpha) and one
// seal (nsnkv_seal_full_tails[_alpha]) over pointers that stay the same from step to
// step.  The plan keeps those pointers and the host copy of the per-sequence counters,
// so a step is one C call with the four per-step pointers: no argument marshalling per
// step in the caller, and the chunk-sizing total (the sum of n_blocks) comes from the
// host counters without reading the device.  It replaces the per-step composition the
// reference drives from Python (the append + restore + SDPA of
// experiments/nb06/source/loop_kv_nb06_attention.py:33-88 followed by post_decode,
// experiments/nb06/source/loop_kv_nb06_packed.py:54-56) for the seal-at-64 policy.
#include <cstdint>
#include <cstring>
#include <new>

#include <cuda_runtime.h>

#include "nsnkv.h"

namespace {

// Staging of nsnkv_paged_step_host: two device slots (a step's q | k_new | v_new in, its
// output out) and two copy streams, made at the first host-buffer step.  Step i uses slot
// i & 1, so the copy of step i + 1's inputs overlaps step i's kernels and the copy of step
// i's output overlaps step i + 1's.
struct HostIo {
  int device = -1;
  uint8_t *slot_in[2] = {nullptr, nullptr};
  uint8_t *slot_out[2] = {nullptr, nullptr};
  cudaStream_t in = nullptr, out = nullptr;
  cudaEvent_t mark[2] = {nullptr, nullptr};   // the caller's stream at a call's entry
  cudaEvent_t ready[2] = {nullptr, nullptr};  // slot inputs copied in
  cudaEvent_t done[2] = {nullptr, nullptr};   // the step's kernels finished with the slot
  cudaEvent_t back[2] = {nullptr, nullptr};   // slot output copied out
  int64_t calls = 0;
};

struct PagedPlan {
  nsnkv_paged_desc d;
  int64_t magic;
  int last_launches;  // kernels the last step launched
  HostIo *io;
};

constexpr int64_t kPlanMagic = 0x6e736e6b7670706cLL;  // "nsnkvppl"
constexpr int kBlock = 64;

PagedPlan *plan_of(void *p) {
  PagedPlan *plan = static_cast<PagedPlan *>(p);
  return plan && plan->magic == kPlanMagic ? plan : nullptr;
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int64_t elem_bytes(const nsnkv_paged_desc &d) { return d.dtype == NSNKV_F16 || d.dtype == NSNKV_BF16 ? 2 : 4; }
int64_t in_bytes(const nsnkv_paged_desc &d) { return d.batch * (d.hq + 2LL * d.h) * 128 * elem_bytes(d); }
int64_t out_bytes(const nsnkv_paged_desc &d) { return d.batch * d.hq * 128LL * elem_bytes(d); }

void free_io(HostIo *io) {
  if (!io) return;
  if (io->in) cudaStreamSynchronize(io->in);
  if (io->out) cudaStreamSynchronize(io->out);
  for (int j = 0; j < 2; ++j) {
    if (io->slot_in[j]) cudaFree(io->slot_in[j]);
    if (io->slot_out[j]) cudaFree(io->slot_out[j]);
    for (cudaEvent_t e : {io->mark[j], io->ready[j], io->done[j], io->back[j]})
      if (e) cudaEventDestroy(e);
  }
  if (io->in) cudaStreamDestroy(io->in);
  if (io->out) cudaStreamDestroy(io->out);
  delete io;
}

// The staging of a plan on the current device, made at its first use.
int make_io(PagedPlan *plan) {
  HostIo *io = new (std::nothrow) HostIo;
  if (!io) return NSNKV_ERR_CUDA;
  bool ok = cudaGetDevice(&io->device) == cudaSuccess;
  ok = ok && cudaStreamCreateWithFlags(&io->in, cudaStreamNonBlocking) == cudaSuccess;
  ok = ok && cudaStreamCreateWithFlags(&io->out, cudaStreamNonBlocking) == cudaSuccess;
  for (int j = 0; j < 2 && ok; ++j) {
    ok = cudaMalloc(&io->slot_in[j], in_bytes(plan->d)) == cudaSuccess &&
         cudaMalloc(&io->slot_out[j], out_bytes(plan->d)) == cudaSuccess;
    for (cudaEvent_t *e : {&io->mark[j], &io->ready[j], &io->done[j], &io->back[j]})
      ok = ok && cudaEventCreateWithFlags(e, cudaEventDisableTiming) == cudaSuccess;
  }
  if (!ok) {
    free_io(io);
    return NSNKV_ERR_CUDA;
  }
  plan->io = io;
  return NSNKV_OK;
}

}  // namespace

namespace nsnkv {
int attn_last_launches();  // attention.cu: kernels of the calling thread's last decode call
}

extern "C" {

int nsnkv_paged_plan_create(const nsnkv_paged_desc *desc, void **plan_out) {
  if (!desc || !plan_out) return NSNKV_ERR_ARG;
  *plan_out = nullptr;
  if (desc->struct_bytes != static_cast<int64_t>(sizeof(nsnkv_paged_desc))) return NSNKV_ERR_ARG;
  const nsnkv_paged_desc &d = *desc;
  if (d.batch <= 0 || d.h <= 0 || d.hq <= 0 || d.hq % d.h != 0 || d.max_blocks <= 0) return NSNKV_ERR_ARG;
  if (d.bits < 3 || d.bits > 5 || (d.dtype != NSNKV_F16 && d.dtype != NSNKV_BF16)) return NSNKV_ERR_ARG;
  if (d.flags & ~(NSNKV_ATTN_RECORD_ORDER | NSNKV_ATTN_EXACT)) return NSNKV_ERR_ARG;
  if (!d.k_codes || !d.k_norm || !d.k_min || !d.k_scale || !d.v_codes || !d.v_norm || !d.v_min || !d.v_scale)
    return NSNKV_ERR_ARG;
  if ((d.k_alpha == nullptr) != (d.v_alpha == nullptr)) return NSNKV_ERR_ARG;
  if (d.flags && !d.k_alpha) return NSNKV_ERR_ARG;  // record orders and exact attention need the factors
  if (!d.block_table || d.table_stride < d.max_blocks || !d.n_blocks || !d.tail_len) return NSNKV_ERR_ARG;
  if (!d.k_tail || !d.v_tail || d.tail_stride_head < kBlock || d.tail_stride_seq < d.h * d.tail_stride_head)
    return NSNKV_ERR_ARG;
  if (!d.workspace || d.workspace_bytes < nsnkv_decode_attn_workspace_bytes(d.batch, d.hq, d.h, d.max_blocks,
                                                                            kBlock - 1))
    return NSNKV_ERR_ARG;
  if (!d.status || !d.host_n_blocks || !d.host_tail_len) return NSNKV_ERR_ARG;
  if (!aligned(d.host_n_blocks, 4) || !aligned(d.host_tail_len, 4)) return NSNKV_ERR_ARG;
  for (int64_t b = 0; b < d.batch; ++b) {
    const int32_t nb = d.host_n_blocks[b], tl = d.host_tail_len[b];
    if (nb < 0 || nb > d.max_blocks || tl < 0 || tl >= kBlock) return NSNKV_ERR_ARG;
  }
  PagedPlan *plan = new (std::nothrow) PagedPlan;
  if (!plan) return NSNKV_ERR_CUDA;
  std::memcpy(&plan->d, desc, sizeof(nsnkv_paged_desc));
  plan->magic = kPlanMagic;
  plan->last_launches = 0;
  plan->io = nullptr;
  *plan_out = plan;
  return NSNKV_OK;
}

int nsnkv_paged_step(void *plan_handle, const void *q, const void *k_new, const void *v_new, void *out,
                     void *attn_event, void *stream) {
  PagedPlan *plan = plan_of(plan_handle);
  if (!plan || !q || !k_new || !v_new || !out) return NSNKV_ERR_ARG;
  const nsnkv_paged_desc &d = plan->d;
  int64_t total = 0;
  for (int64_t b = 0; b < d.batch; ++b) {
    // the appended token lands at tail index tail_len[b], which must leave a free row
    if (d.host_n_blocks[b] >= d.max_blocks && d.host_tail_len[b] + 1 >= kBlock) return NSNKV_ERR_TOO_LARGE;
    total += d.host_n_blocks[b];
  }
  int rc = nsnkv_decode_attn_alpha(
      d.batch, d.hq, d.h, d.bits, d.dtype, q, d.k_codes, d.k_norm, d.k_min, d.k_scale, d.v_codes, d.v_norm, d.v_min,
      d.v_scale, d.k_alpha, d.v_alpha, d.blk_bytes, d.flags, d.blk_stride_head, d.blk_stride_page, d.block_table,
      d.table_stride, d.n_blocks, 0, d.max_blocks, total, d.k_tail, d.v_tail, d.tail_stride_seq, d.tail_stride_head,
      d.tail_len, 0, kBlock - 1, k_new, v_new, out, nullptr, nullptr, d.workspace, d.workspace_bytes, d.status,
      stream);
  if (rc != NSNKV_OK) return rc;
  const int attn_launches = nsnkv::attn_last_launches();
  if (attn_event && cudaEventRecord(static_cast<cudaEvent_t>(attn_event), static_cast<cudaStream_t>(stream)) !=
                        cudaSuccess)
    return NSNKV_ERR_CUDA;
  if (d.k_alpha)
    rc = nsnkv_seal_full_tails_alpha(
        d.batch, d.h, d.bits, d.dtype, d.k_tail, d.v_tail, d.tail_stride_seq, d.tail_stride_head, d.tail_len,
        d.n_blocks, 1, d.block_table, d.table_stride, d.k_codes, d.k_norm, d.k_min, d.k_scale, d.v_codes, d.v_norm,
        d.v_min, d.v_scale, d.k_alpha, d.v_alpha, d.blk_bytes, (d.flags & NSNKV_ATTN_RECORD_ORDER) ? 1 : 0,
        d.seq_counters, d.blk_stride_head, d.blk_stride_page, d.status, stream);
  else
    rc = nsnkv_seal_full_tails(d.batch, d.h, d.bits, d.dtype, d.k_tail, d.v_tail, d.tail_stride_seq,
                               d.tail_stride_head, d.tail_len, d.n_blocks, 1, d.block_table, d.table_stride,
                               d.k_codes, d.k_norm, d.k_min, d.k_scale, d.v_codes, d.v_norm, d.v_min, d.v_scale,
                               d.blk_stride_head, d.blk_stride_page, d.status, stream);
  if (rc != NSNKV_OK) return rc;
  // the seal is one launch, two without the per-sequence counters (a counter kernel follows)
  plan->last_launches = attn_launches + (d.k_alpha && d.seq_counters ? 1 : 2);
  // the seal-at-64 policy is deterministic: every tail grows by one and a full one seals
  for (int64_t b = 0; b < d.batch; ++b) {
    const int32_t t = d.host_tail_len[b] + 1;
    if (t >= kBlock) {
      d.host_n_blocks[b] += 1;
      d.host_tail_len[b] = t - kBlock;
    } else {
      d.host_tail_len[b] = t;
    }
  }
  return NSNKV_OK;
}

int nsnkv_paged_step_host(void *plan_handle, const void *host_in, void *host_out, void *done_event,
                          void *stream) {
  PagedPlan *plan = plan_of(plan_handle);
  if (!plan || !host_in || !host_out) return NSNKV_ERR_ARG;
  const nsnkv_paged_desc &d = plan->d;
  for (int64_t b = 0; b < d.batch; ++b)  // checked before anything is enqueued
    if (d.host_n_blocks[b] >= d.max_blocks && d.host_tail_len[b] + 1 >= kBlock) return NSNKV_ERR_TOO_LARGE;
  if (!plan->io) {
    const int rc = make_io(plan);
    if (rc != NSNKV_OK) return rc;
  }
  HostIo &io = *plan->io;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != io.device) return NSNKV_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int j = static_cast<int>(io.calls & 1);
  const int64_t nq = d.batch * d.hq * 128LL * elem_bytes(d), nk = d.batch * d.h * 128LL * elem_bytes(d);
  // inputs: after the caller's stream reached the previous call (the first call: this one),
  // and after step i - 2 finished reading the slot
  bool ok = cudaEventRecord(io.mark[j], st) == cudaSuccess;
  ok = ok && cudaStreamWaitEvent(io.in, io.mark[io.calls ? j ^ 1 : j], 0) == cudaSuccess;
  if (io.calls >= 2) ok = ok && cudaStreamWaitEvent(io.in, io.done[j], 0) == cudaSuccess;
  ok = ok && cudaMemcpyAsync(io.slot_in[j], host_in, in_bytes(d), cudaMemcpyHostToDevice, io.in) == cudaSuccess;
  ok = ok && cudaEventRecord(io.ready[j], io.in) == cudaSuccess;
  // the step: after its inputs landed and step i - 2's output left the slot
  ok = ok && cudaStreamWaitEvent(st, io.ready[j], 0) == cudaSuccess;
  if (io.calls >= 2) ok = ok && cudaStreamWaitEvent(st, io.back[j], 0) == cudaSuccess;
  if (!ok) return NSNKV_ERR_CUDA;
  const uint8_t *in = io.slot_in[j];
  const int rc = nsnkv_paged_step(plan_handle, in, in + nq, in + nq + nk, io.slot_out[j], nullptr, stream);
  if (rc != NSNKV_OK) return rc;
  // the output: back to host memory once the step's kernels finished
  ok = cudaEventRecord(io.done[j], st) == cudaSuccess;
  ok = ok && cudaStreamWaitEvent(io.out, io.done[j], 0) == cudaSuccess;
  ok = ok && cudaMemcpyAsync(host_out, io.slot_out[j], out_bytes(d), cudaMemcpyDeviceToHost, io.out) == cudaSuccess;
  ok = ok && cudaEventRecord(io.back[j], io.out) == cudaSuccess;
  if (done_event) ok = ok && cudaEventRecord(static_cast<cudaEvent_t>(done_event), io.out) == cudaSuccess;
  io.calls += 1;
  return ok ? NSNKV_OK : NSNKV_ERR_CUDA;
}

int nsnkv_paged_plan_last_launches(void *plan_handle) {
  const PagedPlan *plan = plan_of(plan_handle);
  return plan ? plan->last_launches : NSNKV_ERR_ARG;
}

int nsnkv_paged_plan_destroy(void *plan_handle) {
  PagedPlan *plan = plan_of(plan_handle);
  if (!plan) return NSNKV_ERR_ARG;
  plan->magic = 0;
  free_io(plan->io);
  delete plan;
  return NSNKV_OK;
}

}  // extern "C"
