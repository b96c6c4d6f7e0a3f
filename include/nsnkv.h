/*
 * nsnkv.h - C ABI of the B200 (sm_100a) implementation of NSN's packed-KV path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), launches asynchronously on that stream and never
 * synchronises.  Argument errors are returned as negative int codes before
 * anything is launched.  Data errors found on the device (non-finite input,
 * fp16 metadata overflow/underflow, non-finite output) are OR-ed into a caller
 * owned device int32 status word, which the caller reads when it chooses.
 *
 * Block format (identical to the reference codec, bit for bit):
 *   one block = 64 tokens x 128 channels of one (sequence, kv head);
 *   codes  : LSB-first bitstream, element i = token*128 + channel occupies
 *            bits [bits*i, bits*i + bits); 3072 B (INT3) / 4096 B (INT4) /
 *            5120 B (INT5) per block;
 *   norm   : fp16 [64]   per-token L2 norm;
 *   min    : fp16 [128]  per-channel minimum of the unit direction;
 *   scale  : fp16 [128]  per-channel (max - min) / (2^bits - 1);
 *   header : 12 bytes '<QHBB' = token offset u64, 64 u16, bits u8, 0 u8.
 * fp16/bf16 values are passed as raw uint16_t bit patterns.
 */
#ifndef NSNKV_H
#define NSNKV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* return codes */
#define NSNKV_OK 0
#define NSNKV_ERR_ARG (-1)         /* bad size, null pointer, misaligned pointer, bad dtype/bits */
#define NSNKV_ERR_LAUNCH (-2)      /* the CUDA launch itself failed */
#define NSNKV_ERR_UNSUPPORTED (-3) /* valid but not built (e.g. a GQA group size without a kernel) */
#define NSNKV_ERR_CUDA (-4)        /* a CUDA runtime call other than a launch failed */
#define NSNKV_ERR_TOO_LARGE (-5)   /* request exceeds a fixed capacity of the entry point */

/* device status bits (int32, OR-accumulated) */
#define NSNKV_ST_INPUT_NONFINITE 1   /* NaN/Inf in x, q, a tail or a metadata value */
#define NSNKV_ST_META_OVERFLOW 2     /* fp16 norm/min/scale overflowed or is non-finite */
#define NSNKV_ST_META_UNDERFLOW 4    /* a nonzero norm or scale rounded to fp16 zero */
#define NSNKV_ST_OUTPUT_NONFINITE 8  /* NaN/Inf in a reconstruction or attention output */
#define NSNKV_ST_TIMEOUT 32          /* a bounded wait inside a kernel gave up */
#define NSNKV_ST_CAPACITY 64         /* an appended token found its tail buffer full (not stored) */

/* element dtypes */
#define NSNKV_F16 0
#define NSNKV_BF16 1
#define NSNKV_F32 2

int nsnkv_version(void);

/* Bytes of one packed 64x128 block for `bits` (3, 4 or 5); 0 for other values. */
int64_t nsnkv_block_code_bytes(int bits);

/*
 * Encode rows x blocks_per_row contiguous 64x128 blocks of x.
 * Replaces nsn_encode (experiments/nb06/source/loop_kv_nb06_primitives.py:37-55)
 * followed by pack3 / pack_codes (loop_kv_nb06_codec.py:6-15,
 * loop_kv_nb06_primitives.py:15-24) and the header of encode_group
 * (loop_kv_nb06_codec.py:28-34).
 *   x          [rows][blocks_per_row][64][128] of x_dtype, contiguous, 16-byte aligned
 *   norm_order 0: the 8-lane sum-of-squares order torch uses for contiguous
 *              rows; 1: sequential order (torch's order for strided rows)
 *   input block (r, i) is written to output block index
 *              o = r*out_row_stride + out_offset + i  (contiguous when
 *              out_row_stride == blocks_per_row and out_offset == 0)
 *   codes      [o][block_code_bytes] packed output (may be NULL)
 *   q_out      [rows*blocks_per_row][64][128] unpacked uint8 codes in input order (may be NULL)
 *   norm       [o][64] fp16; mn, scale [o][128] fp16
 *   headers    [o][12] (may be NULL); token offset header_start + 64*i
 *   status     device int32, OR-ed with NSNKV_ST_* bits
 */
int nsnkv_encode_blocks(const void *x, int x_dtype, int64_t rows, int64_t blocks_per_row, int bits, int norm_order,
                        uint8_t *codes, uint8_t *q_out, uint16_t *norm, uint16_t *mn, uint16_t *scale,
                        uint8_t *headers, int64_t header_start, int64_t out_row_stride, int64_t out_offset,
                        int32_t *status, void *stream);

/*
 * Block strides.  The paged cache keeps the blocks of INT3 fp16 caches as block
 * records: per (kv head, page) one record of 2 * (code_bytes + 768) bytes (7680 for
 * INT3) holding K codes | K min (128 fp16) | K scale (128 fp16) | K renorm factors
 * (64 fp32), then the same four fields for V; the norms stay in dense arrays.  Entry
 * points that take blk_bytes address block o of the codes, min, scale and factor
 * arrays at base + o * blk_bytes (blk_bytes a multiple of 16, at least code_bytes);
 * blk_bytes = 0 means dense arrays (code_bytes, 256, 256 and 256 bytes per block).
 * Norm arrays are always dense (128 bytes per block).
 *
 * Code orders.  The same packed bytes in three orders (code_order):
 *   0  the reference's rows back to back (LSB-first bitstream, 16*bits bytes per token);
 *   1  paired rows, the V codes of the records: the rows of tokens 2j and 2j+1
 *      interleaved at 16 bits, 32-bit word j*8*bits + k = [row 2j half k | row 2j+1 half k];
 *   2  paired halves, the K codes of the records: in each row, each 32-code group
 *      (2*bits 16-bit halves: A = the first bits, B = the rest) stored as words
 *      [A half m | B half m], m < bits.
 * The tensor-core kernel then reads two codes of one register (two tokens of a channel
 * for V, two channels of a token for K) from the same word.  The decode and seal entry
 * points take rec_order (1: K in order 2 and V in order 1, as in the records; 0: both in
 * order 0); everything without such an argument takes order 0.
 *
 * nsnkv_encode_blocks with block strides: codes, mn and scale are fields of records
 * blk_bytes apart (0: identical to nsnkv_encode_blocks); codes written in code_order.
 */
int nsnkv_encode_blocks_strided(const void *x, int x_dtype, int64_t rows, int64_t blocks_per_row, int bits,
                                int norm_order, uint8_t *codes, uint8_t *q_out, uint16_t *norm, uint16_t *mn,
                                uint16_t *scale, uint8_t *headers, int64_t header_start, int64_t out_row_stride,
                                int64_t out_offset, int64_t blk_bytes, int code_order, int32_t *status, void *stream);

/*
 * Reconstruct rows of sealed blocks followed by an optional native tail.
 * Replaces nsn_decode (loop_kv_nb06_primitives.py:57-66), restore_group
 * (loop_kv_nb06_codec.py:36-38) and the VF01 bridge restore_v/materialize
 * (experiments/ac08/source/loop_kv_vf01_kernel.py:47-54,120-126).
 *   rows x blocks_per_row blocks, block (r, i) at index r*blocks_per_row + i
 *   codes      packed [n][block_code_bytes] (codes_unpacked = 0) or
 *              unpacked uint8 [n][64][128] (codes_unpacked = 1)
 *   tail       [rows][tail_len][128] of dtype (may be NULL when tail_len = 0)
 *   out        [rows][blocks_per_row*64 + tail_len][128] of dtype
 * Bit-exact with the reference's CPU arithmetic (8-lane norm order).
 */
int nsnkv_restore(const uint8_t *codes, int codes_unpacked, const uint16_t *norm, const uint16_t *mn,
                  const uint16_t *scale, int64_t rows, int64_t blocks_per_row, int bits,
                  const void *tail, int64_t tail_len, int dtype, void *out, int32_t *status, void *stream);

/*
 * LSB-first bitstream pack / unpack of `count` codes (any count).
 * Replaces pack_codes / unpack_codes_reference (loop_kv_nb06_primitives.py:15-35)
 * and pack3 / unpack3 (loop_kv_nb06_codec.py:6-26).  pack sets
 * NSNKV_ST_INPUT_NONFINITE in status when a code is >= 2^bits.
 */
int nsnkv_pack(const uint8_t *codes, int64_t count, int bits, uint8_t *out, int32_t *status, void *stream);
int nsnkv_unpack(const uint8_t *payload, int64_t count, int bits, uint8_t *out, void *stream);

/*
 * Fused packed-KV decode attention, one query token per sequence.
 * Replaces VF01/NB06 launch(g, kt, q, vg, vt) (loop_kv_vf01_kernel.py:128-139,
 * experiments/nb06/source/loop_kv_nb06_kernel.py:142-154): _partial + _merge.
 *
 * Sequence b, kv head h attends over n_blocks[b] sealed blocks followed by
 * tail_len[b] native tail tokens (plus the appended token when k_new != NULL).
 * Query head j uses kv head j / (hq / h) (repeat_kv grouping).
 *   q            [batch][hq][128] of dtype
 *   k_*, v_*     block pools; block (b, h, i) has index
 *                  h*blk_stride_head + page*blk_stride_page,
 *                page = block_table ? block_table[b*table_stride + i] : i
 *   n_blocks     per-sequence sealed block count (device, may be NULL: use n_blocks_const)
 *   k_tail/v_tail  element (b, h, j, c) at ((b*tail_stride_seq + h*tail_stride_head + j)*128 + c)
 *   tail_len     per-sequence tail length (device, may be NULL: use tail_len_const)
 *   k_new/v_new  [batch][h][128] token appended at tail index tail_len[b] and
 *                attended (may be NULL); written into the tail buffers
 *   max_blocks   upper bound of n_blocks[b] (sizes the launch grid)
 *   out          [batch][hq][128] of dtype; out_f32 (may be NULL) fp32 copy;
 *   lse          [batch][hq] log-sum-exp of the scaled scores (may be NULL)
 *   workspace    device scratch of nsnkv_decode_attn_workspace_bytes() bytes, 16-byte
 *                aligned, any contents; calls that may run at the same time need
 *                separate ones.
 *                It holds the chunk partials and, first, one 64-bit word per
 *                (sequence, kv head) in which the chunk CTAs count their arrival under
 *                a per-call epoch; with at most 32 chunks per sequence the last CTA to
 *                arrive merges the sequence's partials, and no merge kernel runs.
 * Scores use scale 1/sqrt(128); softmax and accumulation are fp32.
 */
int nsnkv_decode_attn(int64_t batch, int hq, int h, int bits, int dtype, const void *q,
                      const uint8_t *k_codes, const uint16_t *k_norm, const uint16_t *k_min, const uint16_t *k_scale,
                      const uint8_t *v_codes, const uint16_t *v_norm, const uint16_t *v_min, const uint16_t *v_scale,
                      int64_t blk_stride_head, int64_t blk_stride_page,
                      const int32_t *block_table, int64_t table_stride,
                      const int32_t *n_blocks, int32_t n_blocks_const, int32_t max_blocks,
                      void *k_tail, void *v_tail, int64_t tail_stride_seq, int64_t tail_stride_head,
                      const int32_t *tail_len, int32_t tail_len_const, int32_t max_tail,
                      const void *k_new, const void *v_new,
                      void *out, float *out_f32, float *lse,
                      void *workspace, int64_t workspace_bytes, int32_t *status, void *stream);

/*
 * nsnkv_decode_attn over blocks that also carry per-token renorm factors:
 *   k_alpha / v_alpha  fp32 [64] per block, indexed like k_norm / v_norm, holding
 *                      alpha_t = n_t / max(||d_t||, 1e-12) (0 when n_t == 0) with
 *                      d = min + scale * code: the factor nsn_decode applies to a row
 *                      (loop_kv_nb06_primitives.py:57-66); nsnkv_block_renorm and
 *                      nsnkv_seal_full_tails_alpha write it.  Both may be NULL: the
 *                      blocks then take the nsnkv_decode_attn path (with blk_bytes).
 *   blk_bytes          block stride of the codes, min, scale and factor arrays (0: dense;
 *                      see nsnkv_encode_blocks_strided).  When each block's K fields and
 *                      then its V fields form one block record (k_min = k_codes + CB,
 *                      k_scale = k_codes + CB + 256, k_alpha = k_codes + CB + 512,
 *                      v_codes = k_codes + CB + 768, the same offsets from v_codes, and
 *                      blk_bytes = 2 * (CB + 768)), a block moves in one copy.
 *   blocks_total       sum of n_blocks[b] over the batch when the caller knows it (0: not
 *                      known), with n_blocks given; it only sizes the tensor-core kernels'
 *                      chunks (a wrong value costs speed, never correctness).
 *   flags              NSNKV_ATTN_RECORD_ORDER: K and V codes in the records' orders (K
 *                      paired halves, V paired rows); only the tensor-core kernels read
 *                      them (NSNKV_ERR_UNSUPPORTED otherwise).
 *                      NSNKV_ATTN_EXACT: attend over the exact fp32 restore instead of K
 *                      rounded like the bridge (INT3 fp16, hq / h <= 4 only).
 * Default (flags = NSNKV_ATTN_RECORD_ORDER, one block record per block, INT3, fp16 or
 * bf16, hq / h <= 8): the sealed blocks run on the tensor cores.  K rows are restored
 * and rounded to dtype as restore_group(g, dtype) rounds them
 * (loop_kv_nb06_codec.py:36-38), so the scores are those of the reference bridge; V is
 * applied as the exact fp32 restore with the codes as MMA operands (its rounding moves
 * an output by about 2^-12 of its size).  NSNKV_ATTN_EXACT applies K exactly as well.
 * The norms are not read.  Other shapes take the nsnkv_decode_attn path, which rounds
 * both K and V.  Same workspace.
 */
#define NSNKV_ATTN_RECORD_ORDER 1
#define NSNKV_ATTN_EXACT 2
int nsnkv_decode_attn_alpha(int64_t batch, int hq, int h, int bits, int dtype, const void *q,
                            const uint8_t *k_codes, const uint16_t *k_norm, const uint16_t *k_min,
                            const uint16_t *k_scale, const uint8_t *v_codes, const uint16_t *v_norm,
                            const uint16_t *v_min, const uint16_t *v_scale,
                            const float *k_alpha, const float *v_alpha, int64_t blk_bytes, int flags,
                            int64_t blk_stride_head, int64_t blk_stride_page,
                            const int32_t *block_table, int64_t table_stride,
                            const int32_t *n_blocks, int32_t n_blocks_const, int32_t max_blocks,
                            int64_t blocks_total,
                            void *k_tail, void *v_tail, int64_t tail_stride_seq, int64_t tail_stride_head,
                            const int32_t *tail_len, int32_t tail_len_const, int32_t max_tail,
                            const void *k_new, const void *v_new,
                            void *out, float *out_f32, float *lse,
                            void *workspace, int64_t workspace_bytes, int32_t *status, void *stream);

/*
 * Per-token renorm factors of sealed blocks (see nsnkv_decode_attn_alpha), for the
 * blocks nsnkv_encode_blocks lays out: block (row r, i) of rows x blocks_per_row has
 * index r*row_stride + offset + i in codes / norm / min / scale / alpha; blk_bytes is
 * the block stride of codes / min / scale / alpha (0: dense); codes read in code_order.
 */
int nsnkv_block_renorm(int bits, int64_t rows, int64_t blocks_per_row, const uint8_t *codes, const uint16_t *norm,
                       const uint16_t *min, const uint16_t *scale, int64_t row_stride, int64_t offset, float *alpha,
                       int64_t blk_bytes, int code_order, void *stream);

/* Workspace bytes nsnkv_decode_attn needs for these sizes. */
int64_t nsnkv_decode_attn_workspace_bytes(int64_t batch, int hq, int h, int32_t max_blocks, int32_t max_tail);

/*
 * nsnkv_decode_attn without a workspace argument, for callers that cannot allocate
 * device memory: code running where cudaMalloc is not allowed or not wanted (a
 * serving loop that must not call into the allocator or implicitly synchronise the
 * device, a host runtime without access to the framework's caching allocator, an
 * embedding that owns all device memory itself).  This entry point has no
 * counterpart in the reference.
 *
 * Arguments and results are those of nsnkv_decode_attn minus workspace /
 * workspace_bytes.  The split-KV partials live in a fixed device array of
 * NSNKV_NOALLOC_SCRATCH_BYTES (16 MiB) compiled into the library; every GPU that
 * loads the library holds it until the process exits.  Requests whose
 * nsnkv_decode_attn_workspace_bytes() exceed it return NSNKV_ERR_TOO_LARGE
 * (e.g. batch 64 x 32 query heads x 16k-token contexts does not fit; one 32k-token
 * sequence does).  The first call on each device looks up the array's device
 * address with that device current (cudaGetSymbolAddress); make that first call
 * before any stream capture.  No call allocates (no cudaMalloc/cudaFree or any
 * allocating library routine).  All calls share the array and it keeps the last
 * call's contents; nothing in it needs to start at zero, but calls that overlap on
 * the GPU (for example on two streams of the same device) race on it.
 */
#define NSNKV_NOALLOC_SCRATCH_BYTES (16ll << 20)
int nsnkv_decode_attn_noalloc(int64_t batch, int hq, int h, int bits, int dtype, const void *q,
                              const uint8_t *k_codes, const uint16_t *k_norm, const uint16_t *k_min,
                              const uint16_t *k_scale, const uint8_t *v_codes, const uint16_t *v_norm,
                              const uint16_t *v_min, const uint16_t *v_scale,
                              int64_t blk_stride_head, int64_t blk_stride_page,
                              const int32_t *block_table, int64_t table_stride,
                              const int32_t *n_blocks, int32_t n_blocks_const, int32_t max_blocks,
                              void *k_tail, void *v_tail, int64_t tail_stride_seq, int64_t tail_stride_head,
                              const int32_t *tail_len, int32_t tail_len_const, int32_t max_tail,
                              const void *k_new, const void *v_new,
                              void *out, float *out_f32, float *lse, int32_t *status, void *stream);

/*
 * Seal full tails of a paged cache: for every sequence b whose tail holds
 * 64 tokens (after an append), encode the 64x128 tail of each kv head into
 * page block_table[b*table_stride + n_blocks[b]] of the K and V pools, then set
 * tail_len[b] = 0 and n_blocks[b] += 1.  Sequences with shorter tails are left
 * unchanged.  Replaces the per-slot compress_to/post_decode seal
 * (experiments/nb06/source/loop_kv_nb06_packed.py:36-56) with the
 * seal-at-64 policy.  pending_append = 1 counts the token appended by the
 * preceding nsnkv_decode_attn (k_new != NULL) into the tail length.  A sequence
 * whose table row has no page left (n_blocks[b] == table_stride) keeps its full
 * tail and sets NSNKV_ST_CAPACITY; the next append to it is refused the same way.
 */
int nsnkv_seal_full_tails(int64_t batch, int h, int bits, int dtype,
                          void *k_tail, void *v_tail, int64_t tail_stride_seq, int64_t tail_stride_head,
                          int32_t *tail_len, int32_t *n_blocks, int pending_append,
                          const int32_t *block_table, int64_t table_stride,
                          uint8_t *k_codes, uint16_t *k_norm, uint16_t *k_min, uint16_t *k_scale,
                          uint8_t *v_codes, uint16_t *v_norm, uint16_t *v_min, uint16_t *v_scale,
                          int64_t blk_stride_head, int64_t blk_stride_page,
                          int32_t *status, void *stream);

/*
 * nsnkv_seal_full_tails that also writes the sealed blocks' renorm factors
 * (k_alpha / v_alpha, fp32 [64] per block) in the same kernel.  seq_counters
 * (int32 [batch], may be NULL) must be zero before the first call and are left zero:
 * with them the last CTA of each sequence advances n_blocks / tail_len, so the call is
 * one launch; without them a second kernel advances the counters.  blk_bytes is the
 * block stride of the codes / min / scale / alpha arrays (0: dense); rec_order = 1 writes
 * the codes in the records' orders (K paired halves, V paired rows).
 */
int nsnkv_seal_full_tails_alpha(int64_t batch, int h, int bits, int dtype,
                                void *k_tail, void *v_tail, int64_t tail_stride_seq, int64_t tail_stride_head,
                                int32_t *tail_len, int32_t *n_blocks, int pending_append,
                                const int32_t *block_table, int64_t table_stride,
                                uint8_t *k_codes, uint16_t *k_norm, uint16_t *k_min, uint16_t *k_scale,
                                uint8_t *v_codes, uint16_t *v_norm, uint16_t *v_min, uint16_t *v_scale,
                                float *k_alpha, float *v_alpha, int64_t blk_bytes, int rec_order, int32_t *seq_counters,
                                int64_t blk_stride_head, int64_t blk_stride_page, int32_t *status, void *stream);

/*
 * Decode-step plan over a paged cache with the seal-at-64 policy.  One step is
 * nsnkv_decode_attn_alpha (append k_new / v_new, attend with q; max_tail 63,
 * blocks_total from the host counters) followed by nsnkv_seal_full_tails_alpha
 * (pending_append 1; nsnkv_seal_full_tails when the pools carry no renorm factors),
 * over the pointers of the descriptor, which the plan copies.  Together they replace
 * the reference's per-step append + attention + post_decode
 * (experiments/nb06/source/loop_kv_nb06_attention.py:33-88,
 * experiments/nb06/source/loop_kv_nb06_packed.py:54-56).
 *   struct_bytes     sizeof(nsnkv_paged_desc) as the caller laid it out
 *   flags            nsnkv_decode_attn_alpha flags (they need k_alpha / v_alpha)
 *   tail buffers     64 rows per (sequence, kv head): tail_stride_head >= 64
 *   workspace        >= nsnkv_decode_attn_workspace_bytes(batch, hq, h, max_blocks, 63)
 *   seq_counters     as for nsnkv_seal_full_tails_alpha (may be NULL)
 *   host_n_blocks / host_tail_len  int32 [batch] in host memory, equal to the device
 *                    counters when the plan is made; the plan reads them for the
 *                    chunk sizing and advances them in place after every step, so they
 *                    stay equal to the device counters without a device read.  They
 *                    must outlive the plan.
 * attn_event (a cudaEvent_t, may be NULL) is recorded on the stream between the attention
 * launches and the seal, for timing the two apart.
 * nsnkv_paged_step returns NSNKV_ERR_TOO_LARGE, launching nothing, when a sequence
 * would need a page beyond max_blocks.  A plan is used by one thread at a time; all
 * the memory it names stays owned by the caller.
 */
typedef struct nsnkv_paged_desc {
  int64_t struct_bytes;
  int64_t batch;
  int32_t hq, h, bits, dtype;
  int32_t flags, max_blocks;
  uint8_t *k_codes;
  uint16_t *k_norm, *k_min, *k_scale;
  float *k_alpha;
  uint8_t *v_codes;
  uint16_t *v_norm, *v_min, *v_scale;
  float *v_alpha;
  int64_t blk_bytes, blk_stride_head, blk_stride_page;
  const int32_t *block_table;
  int64_t table_stride;
  int32_t *n_blocks, *tail_len;
  void *k_tail, *v_tail;
  int64_t tail_stride_seq, tail_stride_head;
  int32_t *seq_counters;
  void *workspace;
  int64_t workspace_bytes;
  int32_t *status;
  int32_t *host_n_blocks, *host_tail_len;
} nsnkv_paged_desc;
int nsnkv_paged_plan_create(const nsnkv_paged_desc *desc, void **plan);
int nsnkv_paged_step(void *plan, const void *q, const void *k_new, const void *v_new, void *out,
                     void *attn_event, void *stream);
/*
 * One step with host buffers: host_in holds the step's q [batch, hq, 128], k_new and
 * v_new [batch, h, 128] back to back in the cache dtype; host_out receives the output
 * [batch, hq, 128].  The plan copies host_in into one of two device slots on a copy
 * stream of its own, runs nsnkv_paged_step on `stream` over that slot, and copies the
 * output back on a second copy stream; with pinned host buffers the copies of
 * neighbouring steps overlap this step's kernels.  The input copy starts once `stream`
 * reached the previous host-buffer call (the first call: this one).  done_event (a
 * cudaEvent_t, may be NULL) is recorded after the output copy: host_out is written, and
 * host_in may be reused, once it completed.  The slots and streams are made on the
 * current device at the first call (later calls on another device: NSNKV_ERR_ARG) and
 * released by nsnkv_paged_plan_destroy, which first waits for the plan's copies.
 * Replaces the caller-side staging of the reference's decode step (its tensors move
 * to the device inside the HF forward,
 * experiments/nb06/source/loop_kv_nb06_attention.py:33-88).
 */
int nsnkv_paged_step_host(void *plan, const void *host_in, void *host_out, void *done_event, void *stream);
/* Kernels the plan's last successful step launched (0 before the first step). */
int nsnkv_paged_plan_last_launches(void *plan);
int nsnkv_paged_plan_destroy(void *plan);

/*
 * Fused per-token layer ops of a decoder's decode step (nsn_b200/looped.py), in the
 * rounding order of the transformers Llama modules the reference's model adapter drives
 * (experiments/ac08/source/loop_kv_ac08_attention.py:46-96).  Rows are contiguous, dtype
 * NSNKV_F16 or NSNKV_BF16.
 *   nsnkv_add_rmsnorm  residual_out = x + residual (residual may be NULL: x itself, and
 *                      residual_out may then be NULL), out = weight * RMSNorm(residual_out)
 *                      with fp32 statistics (LlamaRMSNorm); dim <= 8192
 *   nsnkv_rope_split   one fused projection row [q (hq*128) | k (h*128) | v (h*128)] ->
 *                      RoPE'd q [rows][hq][128], k [rows][h][128] and v [rows][h][128]
 *                      (apply_rotary_pos_emb); cos / sin [128] per row, cs_stride elements
 *                      apart (0: one position for every row)
 *   nsnkv_swiglu       one fused row [gate (inter) | up (inter)] -> silu(gate) * up (LlamaMLP)
 *   nsnkv_gemv_rows    the projections on those few rows: each weight row streams from HBM
 *                      once into tensor-core MMAs
 * All four launch with programmatic dependent launch: a kernel may become resident while
 * the kernel before it on the stream finishes, and waits for it (griddepcontrol.wait)
 * before reading anything; stream order is kept.
 */
int nsnkv_add_rmsnorm(int64_t rows, int dim, int dtype, const void *x, const void *residual, const void *weight,
                      float eps, void *residual_out, void *out, void *stream);
int nsnkv_rope_split(int64_t rows, int hq, int h, int dtype, const void *qkv, const void *cos, const void *sin,
                     int64_t cs_stride, void *q, void *k, void *v, void *stream);
int nsnkv_swiglu(int64_t rows, int inter, int dtype, const void *gate_up, void *out, void *stream);
/* y [m][n] = x [m][k] . w [n][k]^T with fp32 accumulation, for decode rows: m <= 8, n % 8 == 0,
 * k % 256 == 0, x and w 16-byte aligned (a torch Linear without bias on a few rows).
 * flags: NSNKV_GEMV_FIXED_WEIGHTS when no work enqueued on the stream before this call
 * writes w (model weights while decoding): the first weight loads then start before the
 * wait for the preceding kernel, overlapping it; x is read after the wait either way. */
#define NSNKV_GEMV_FIXED_WEIGHTS 1
int nsnkv_gemv_rows(int m, int n, int k, int dtype, const void *x, const void *w, void *y, int flags, void *stream);

/*
 * Combine per-shard attention partials (one row per shard) into the final
 * output: out = sum_s exp(lse_s - L) * o_s with L = log sum_s exp(lse_s).
 *   o [n_shards][rows][128] fp32, lse [n_shards][rows] fp32, out [rows][128] of dtype.
 * Used by the sequence-split (split-KV) multi-GPU path after an all-gather.
 */
int nsnkv_merge_shards(int n_shards, int64_t rows, const float *o, const float *lse, int dtype,
                       void *out, float *out_f32, float *lse_out, int32_t *status, void *stream);

/*
 * The same combine over packed per-shard records, the form one all-gather returns:
 * record s starts at records + s * record_stride (floats) and holds o [rows][128]
 * followed by lse [rows].  record_stride >= rows * 129.
 */
int nsnkv_merge_shard_records(int n_shards, int64_t rows, const float *records, int64_t record_stride, int dtype,
                              void *out, float *out_f32, float *lse_out, int32_t *status, void *stream);

/*
 * The split-KV record exchange over peer memory, fused with the merge (replaces the
 * NCCL all-gather + nsnkv_merge_shard_records pair).  Every rank owns an area of
 * nsnkv_peer_area_words(world, hq) fp32 words that every other rank has mapped
 * (symmetric memory): peer_areas is a device array of the world ranks' area addresses
 * as this rank sees them, area this rank's own.  Areas and epochs [hq] (uint32, this
 * rank's) are zero before the first call on every rank, and every rank calls with the
 * same world and hq, once per decode step.  record is this rank's [o (hq x 128) | lse (hq)].
 * The kernel writes its record into every peer's area, waits (bounded, about a second;
 * NSNKV_ST_TIMEOUT and no output on expiry) until every rank's record has arrived in
 * its own, and writes the merged out [hq][128] (out_f32 / lse_out may be NULL).
 */
int64_t nsnkv_peer_area_words(int world, int hq);
int nsnkv_peer_merge_records(int world, int rank, int hq, int dtype, const float *record, void *const *peer_areas,
                             float *area, uint32_t *epochs, void *out, float *out_f32, float *lse_out,
                             int32_t *status, void *stream);

/*
 * Int3AsymNsepPchanCache (src/nsn/cache.py:134-313, from_fp16 / to_fp16): x is
 * [rows][tokens][dim] (dim % 8 == 0, 8 <= dim <= 256, rows <= 65535) in x_dtype.
 * Outputs: packed [rows][tokens][3*dim/8] (3-bit indices, 8 per 3 bytes, LSB first:
 * src/nsn/pack.py:85-128), norm fp16 [rows][tokens], d_min / d_step fp16 [rows][dim].
 * norm_order: 0 when the caller's channel axis is contiguous (torch's 8-lane norm),
 * 1 when it is strided (sequential sum), as for nsnkv_encode_blocks.
 * scratch: device memory of nsnkv_int3asym_scratch_bytes(rows, tokens, dim) bytes.
 * Status: NSNKV_ST_INPUT_NONFINITE for a non-finite input (the reference does not check).
 */
int64_t nsnkv_int3asym_scratch_bytes(int64_t rows, int64_t tokens, int dim);
int nsnkv_int3asym_encode(const void *x, int x_dtype, int64_t rows, int64_t tokens, int dim, int norm_order,
                          uint8_t *packed, uint16_t *norm, uint16_t *d_min, uint16_t *d_step, void *scratch,
                          int64_t scratch_bytes, int32_t *status, void *stream);
/* to_fp16: out fp16 [rows][tokens][dim] from the fields above. */
int nsnkv_int3asym_decode(const uint8_t *packed, const uint16_t *norm, const uint16_t *d_min, const uint16_t *d_step,
                          int64_t rows, int64_t tokens, int dim, uint16_t *out, void *stream);

/*
 * Batched GQA decode scores over a per-channel quantised K cache, the K1c layout
 * (experiments/kernels/phase_k1c_triton_fused_kernel.py:172-250, triton_decode_scores):
 *   recipe 0 FP16: code is K itself, fp16 [batch][tokens][n_kv*head_dim];
 *   recipe 1 KIVI / 2 NSN: code uint8 [batch][tokens][n_kv*head_dim], k_min / k_step fp16
 *   [batch][n_kv*head_dim]; NSN also eff_norm fp16 [batch][n_kv][tokens].
 * q fp16 [batch][n_q][head_dim]; scores fp32 [batch][n_q][tokens] =
 *   (1/sqrt(head_dim)) * eff_norm * sum_d q * (code * step + min).
 * Contiguous layouts; head_dim % 16 == 0, <= 256; n_q / n_kv <= 8; code 16-byte aligned.
 */
int nsnkv_k1c_scores(int recipe, int64_t batch, int n_q, int n_kv, int64_t tokens, int head_dim, const void *q,
                     const void *code, const uint16_t *k_min, const uint16_t *k_step, const uint16_t *eff_norm,
                     float *scores, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* NSNKV_H */
