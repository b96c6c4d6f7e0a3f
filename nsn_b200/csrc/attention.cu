// Fused packed-KV decode attention for sm_100a (split-KV, flash-decoding style).
//
// One CTA owns (chunk of up to 8 sealed blocks | up to 512 native rows, kv head h,
// sequence b) and serves all G = hq/h <= 8 query heads of that kv head, so every packed
// byte is read from HBM exactly once (the reference's NB06 _partial re-reads each kv
// block G times, experiments/nb06/source/loop_kv_nb06_kernel.py:54-114).
//
// Warp roles (14 warps):
//   producer (warp 12)  TMA bulk copies (cp.async.bulk) of each block's codes and fp16
//                       metadata into a 6-stage ring, then the block's fp32 restore
//                       coefficients; mbarriers full / ready / empty.
//   restore (warps 0-7) warp w restores channels 32(w%4)..+31 of tokens 32(w/4)..+31 (lane =
//                       token, so the channel group's coefficients are warp-uniform loads):
//                       d = min + scale*code (fp32), the row's sum of squares from the four
//                       warps of its token half, k = (norm / max(||d||, eps)) * d rounded to
//                       the bridge dtype -- the value restore_group stores -- written into a
//                       shared tile in the tensor core's no-swizzle operand layout.
//   MMA (warp 13)       one thread issues tcgen05.mma: scores D1 = K . Q^T (M = 64 tokens,
//                       N = 8 heads, TMEM, double buffered) and, later, D2 += V^T . P^T
//                       (M = 128 channels, N = 16: 8 heads of P rounded to the bridge dtype
//                       + 8 heads of its remainder, so the weights keep fp32 accuracy).
//   softmax (warps 8-11) warp 8+q reads the scores of tokens 16q..16q+15 out of TMEM
//                       (lanes 0..15 of TMEM quadrant q) and builds their P rows.
// Each chunk runs in two phases: all K blocks first (scores kept in shared memory and
// the exact chunk maximum found), then all V blocks with P = exp(s - max) at that
// final maximum, so the TMEM accumulator is never rescaled.  The chunk's (o, max, sum)
// partial is combined with the others by the merge kernel (log-sum-exp, the reference's
// merge, loop_kv_af01_kernel.py:70-84).
#include <mutex>
#include <type_traits>

#include "nsnkv_common.cuh"

namespace nsnkv {

struct AttnArgs {
  int64_t batch;
  int hq, h;
  const void *q;
  const uint8_t *kc;
  const uint16_t *kn, *km, *ks;
  const uint8_t *vc;
  const uint16_t *vn, *vm, *vs;
  int64_t sh, sp;
  const int32_t *table;
  int64_t table_stride;
  const int32_t *nblk;
  int32_t nblk_const;
  void *kt, *vt;
  int64_t tss, tsh;
  const int32_t *tlen;
  int32_t tlen_const;
  const void *knew, *vnew;
  int32_t chunk_blocks;
  int32_t max_chunks;
  float *part_o;   // [batch][hq][max_chunks][128]
  float *part_ml;  // [batch][hq][max_chunks][2]
  int32_t *status;
};

constexpr int kHeads = 8;                  // query heads of one kv head (G <= 8)
constexpr int kMetaRow = kDim + kDim / 8;  // fp32 coefficient row padded every 32 channels by 4 floats
constexpr int kRestoreWarps = 8;           // warp w: channel group w%4 of tokens 32(w/4)..32(w/4)+31
constexpr int kSoftmaxWarp0 = 8;           // warps 8..11: warp % 4 = TMEM quadrant of its tokens
constexpr int kSoftmaxWarps = 4;
constexpr int kProducerWarp = 12;
constexpr int kMmaWarp = 13;
constexpr int kThreads = 14 * 32;
constexpr int kStages = 6;                 // TMA ring depth
constexpr int kChunk = 8;                  // 64-token units per chunk (and phase)
constexpr int kTmemCols = 32;              // scores at columns [0, 8) and [8, 16), P.V accumulator at [16, 32)
constexpr int kScRow = kChunk * kBlock + 4;  // padded score row: the 8 heads' rows start in distinct banks

// One block (K or V) as staged by the producer.  The restore coefficients: a code k is
// dropped into mantissa bits [p, p+BITS) of 1.0f, giving x = 1 + k*2^(p-23); then
//   d = min + scale*k = b*x + a,   b = scale * 2^(23-p),   a = min - b.
template <int BITS>
struct Stage {
  uint8_t codes[code_bytes(BITS)];
  uint16_t norm[kBlock];
  uint16_t mn[kDim];
  uint16_t sc[kDim];
  float fa[kMetaRow];
  float fb[kMetaRow];
};

template <int BITS>
struct AttnSmem {
  Stage<BITS> stage[kStages];
  // Restored K tiles are the B operand of Q.K^T (K-major: element (token t, channel c)
  // at byte (t/8)*2048 + (c/8)*128 + (t%8)*16 + (c%8)*2); V tiles the A operand of
  // V^T.P^T (MN-major: byte (c/8)*1024 + (t/8)*128 + (t%8)*16 + (c%8)*2).
  alignas(128) uint16_t tile[2][kBlock * kDim];
  // P, B operand of V^T.P^T (MN-major, N = 16: heads 0..7 P in the bridge dtype, 8..15 the
  // remainder): element (row n, token t) at byte (n/8)*1024 + (t/8)*128 + (t%8)*16 + (n%8)*2,
  // so one token's 8 heads are 16 contiguous bytes.
  alignas(128) uint16_t ptile[2][16 * kBlock];
  // q rows of this kv head, B operand of K.Q^T (K-major, N = 8): byte (c/8)*128 + g*16 + (c%8)*2.
  alignas(128) uint16_t qtile[8 * kDim];
  alignas(16) float scores[kHeads][kScRow];
  float red[kSoftmaxWarps][kHeads];  // per-warp head maxima / sums of the softmax warps
  float ssp[2][4][kBlock];           // per unit parity: sum-of-squares partial of each channel group
  uint64_t full[kStages], ready[kStages], empty[kStages];
  uint64_t tfull[2], tempty[2], pfull[2], pempty[2], d1full[2], d1empty[2];
  uint64_t d2full, done;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ int meta_index(int c) { return c + (c >> 5) * 4; }

// Mantissa position of code j (0..31 within a lane's 32-channel group).  INT3 codes
// are handled in pairs: one shift puts code 2m at bits 17..19 and code 2m+1 at
// 20..22, and two masks turn them into two floats.
template <int BITS>
__host__ __device__ constexpr int code_pos(int j) {
  return BITS == 3 ? ((j & 1) ? 20 : 17) : 23 - BITS;
}

// Round a float pair to the bridge dtype and pack it (low half = .x).
template <typename T> __device__ __forceinline__ uint32_t pack2(float2 v);
template <> __device__ __forceinline__ uint32_t pack2<__half>(float2 v) {
  __half2 h = __float22half2_rn(v);
  return *reinterpret_cast<uint32_t *>(&h);
}
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float2 v) {
  __nv_bfloat162 h = __float22bfloat162_rn(v);
  return *reinterpret_cast<uint32_t *>(&h);
}
template <typename T> __device__ __forceinline__ float2 unpack2(uint32_t u) { return Elem<T>::to_f2(u); }

__device__ __forceinline__ bool finite2(float2 v) { return isfinite(v.x) && isfinite(v.y); }

// ----------------------------------------------------------------- tcgen05 / TMEM
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Shared-memory operand descriptor, no swizzle: core matrices of 8 rows x 16 bytes
// stored contiguously; lbo = byte distance of core matrices along K, sbo = along M/N.
// Fields: start>>4 [0,14), lbo>>4 [16,30), sbo>>4 [32,46), version 1 [46,48), layout 0.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor of tcgen05.mma kind::f16 with an fp32 accumulator: D format
// [4,6) = 1, A/B format [7,10)/[10,13) = 0 f16 | 1 bf16, A/B major [15]/[16] (0 K-major,
// 1 MN-major), N>>3 at [17,23), M>>4 at [24,29).
template <typename T>
__host__ __device__ constexpr uint32_t umma_idesc(int m, int n, int a_mn, int b_mn) {
  return (1u << 4) | ((std::is_same<T, __nv_bfloat16>::value ? 1u : 0u) << 7) |
         ((std::is_same<T, __nv_bfloat16>::value ? 1u : 0u) << 10) | (static_cast<uint32_t>(a_mn) << 15) |
         (static_cast<uint32_t>(b_mn) << 16) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// One arrival on bar once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Orders this thread's shared-memory writes before later reads by the tensor core.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Lane i of the warp reads TMEM lane (taddr lane + i), 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Bounded wait that also gives up once another role has timed out (abort flag).  Each
// try sleeps until the phase completes or kTrySleepNs pass; at most kTryWaits tries.
constexpr uint32_t kTrySleepNs = 10000;
constexpr uint32_t kTryWaits = 1u << 15;  // ~0.33 s in all

__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(kTrySleepNs)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity, int32_t *status, volatile int *abort) {
  for (int i = 0; i < 64; ++i)  // short spin first: a sleeping thread resumes late
    if (mbar_try_wait(bar, parity)) return true;
  for (uint32_t i = 0; i < kTryWaits; ++i) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if (*abort) return false;
  }
  *abort = 1;
  set_status(status, NSNKV_ST_TIMEOUT);
  return false;
}

// The packed codes of one lane's 32 channels of one token row.  A row is 4*BITS
// words and a lane's group BITS words, so the group is always word aligned.
template <int BITS>
struct RowCodes {
  uint32_t w[BITS];
  __device__ __forceinline__ void load(const uint8_t *codes, int t, int tig) {
    const uint32_t *p = reinterpret_cast<const uint32_t *>(codes) + t * 4 * BITS + tig * BITS;
#pragma unroll
    for (int i = 0; i < BITS; ++i) w[i] = p[i];
  }
  // The group's bits moved so that bit `pos` lands at bit `dst` (both compile-time).
  __device__ __forceinline__ uint32_t place(int pos, int dst) const {
    const int wi = pos >> 5, bi = pos & 31;
    if (bi == dst) return w[wi];
    if (bi > dst) return __funnelshift_r(w[wi], wi + 1 < BITS ? w[wi + 1] : 0u, bi - dst);
    return __funnelshift_l(wi > 0 ? w[wi - 1] : 0u, w[wi], dst - bi);
  }
  // x for codes 2m and 2m+1 (see Stage).
  __device__ __forceinline__ float2 xpair(int m) const {
    if (BITS == 3) {
      const uint32_t ws = place(6 * m, 17);
      return f2(__uint_as_float((ws & 0x000E0000u) | 0x3F800000u), __uint_as_float((ws & 0x00700000u) | 0x3F800000u));
    }
    constexpr int p = 23 - BITS;
    constexpr uint32_t mask = ((1u << BITS) - 1u) << p;
    const uint32_t w0 = place(BITS * 2 * m, p), w1 = place(BITS * (2 * m + 1), p);
    return f2(__uint_as_float((w0 & mask) | 0x3F800000u), __uint_as_float((w1 & mask) | 0x3F800000u));
  }
};

// norm / max(||d||, eps) from the row sum of squares (0 when the stored norm is 0).
__device__ __forceinline__ float renorm(float n, float ss) {
  return n == 0.f ? 0.f : (ss > 1e-24f ? n * rsqrtf(ss) : n * 1e12f);
}

// This lane's 32 channels (group cg) of token t: d = min + scale*code (fp32, pairs) and
// their sum of squares.
template <int BITS>
__device__ __forceinline__ float restore_part(const uint8_t *codes, const float *ma, const float *mb, int mi, int t,
                                              int cg, float2 (&d)[16]) {
  RowCodes<BITS> rc;
  rc.load(codes, t, cg);
  float2 s0 = f2(0.f, 0.f), s1 = f2(0.f, 0.f);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 a4 = *reinterpret_cast<const float4 *>(&ma[mi + 4 * q]);
    const float4 b4 = *reinterpret_cast<const float4 *>(&mb[mi + 4 * q]);
    d[2 * q] = __ffma2_rn(f2(b4.x, b4.y), rc.xpair(2 * q), f2(a4.x, a4.y));
    d[2 * q + 1] = __ffma2_rn(f2(b4.z, b4.w), rc.xpair(2 * q + 1), f2(a4.z, a4.w));
    s0 = __ffma2_rn(d[2 * q], d[2 * q], s0);
    s1 = __ffma2_rn(d[2 * q + 1], d[2 * q + 1], s1);
  }
  return (s0.x + s1.x) + (s0.y + s1.y);
}

// k = al * d rounded to the bridge dtype; out packs channel pairs.
template <typename T>
__device__ __forceinline__ void restore_finish(const float2 (&d)[16], float al, uint32_t (&out)[16]) {
#pragma unroll
  for (int m = 0; m < 16; ++m) out[m] = pack2<T>(__fmul2_rn(d[m], f2(al, al)));
}

template <typename T>
__device__ __forceinline__ void load_row32(const T *row, int cbase, uint32_t (&out)[16]) {
  const uint4 *p = reinterpret_cast<const uint4 *>(row + cbase);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 v = p[i];
    out[4 * i] = v.x;
    out[4 * i + 1] = v.y;
    out[4 * i + 2] = v.z;
    out[4 * i + 3] = v.w;
  }
}

template <typename T>
__device__ __forceinline__ int check_row32(const uint32_t (&u)[16]) {
  int bad = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) bad |= !finite2(unpack2<T>(u[i]));
  return bad ? NSNKV_ST_INPUT_NONFINITE : 0;
}

__device__ __forceinline__ void store_row32(uint16_t *dst, const uint32_t (&u)[16]) {
  uint4 *p = reinterpret_cast<uint4 *>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = make_uint4(u[4 * i], u[4 * i + 1], u[4 * i + 2], u[4 * i + 3]);
}

template <int BITS, typename T>
__global__ void __launch_bounds__(kThreads, 2) attn_partial_kernel(const AttnArgs a) {
  constexpr int CB = code_bytes(BITS);
  constexpr float kLog2e = 1.4426950408889634f;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  AttnSmem<BITS> &S = *reinterpret_cast<AttnSmem<BITS> *>(smem_raw);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int chunk = blockIdx.x, h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int G = a.hq / a.h;

  const int nb = a.nblk ? a.nblk[b] : a.nblk_const;
  const int tl = a.tlen ? a.tlen[b] : a.tlen_const;
  const int tail_total = tl + (a.knew ? 1 : 0);
  const int n_sealed_chunks = (nb + a.chunk_blocks - 1) / a.chunk_blocks;
  const int raw_per_chunk = a.chunk_blocks * kBlock;
  const int n_chunks = n_sealed_chunks + (tail_total + raw_per_chunk - 1) / raw_per_chunk;
  if (chunk >= n_chunks) return;  // the whole CTA, before any barrier or TMEM allocation
  const bool is_raw = chunk >= n_sealed_chunks;
  int blk0 = 0, raw0 = 0, raw1 = 0, n = 0;
  if (!is_raw) {
    blk0 = chunk * a.chunk_blocks;
    n = min(nb, blk0 + a.chunk_blocks) - blk0;
  } else {
    raw0 = (chunk - n_sealed_chunks) * raw_per_chunk;
    raw1 = min(tail_total, raw0 + raw_per_chunk);
    n = (raw1 - raw0 + kBlock - 1) / kBlock;
  }
  const int units = 2 * n;  // K units 0..n-1, then V units n..2n-1
  volatile int *abort = &S.abort;
  int st = 0;

  // ---- set-up: barriers, TMEM, the q operand
  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&S.full[i], 1);
      mbar_init(&S.ready[i], 1);
      mbar_init(&S.empty[i], kRestoreWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.tfull[i], kRestoreWarps);
      mbar_init(&S.tempty[i], 1);
      mbar_init(&S.pfull[i], kSoftmaxWarps);
      mbar_init(&S.pempty[i], 1);
      mbar_init(&S.d1full[i], 1);
      mbar_init(&S.d1empty[i], kSoftmaxWarps);
    }
    mbar_init(&S.d2full, 1);
    mbar_init(&S.done, 1);
    S.abort = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&S.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp == kSoftmaxWarp0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int pc = lane + 32 * i, r = pc & 7, c8 = pc >> 3;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (r < G) {
        v = *reinterpret_cast<const uint4 *>(static_cast<const T *>(a.q) + ((b * a.hq) + h * G + r) * kDim + 8 * c8);
        if (!finite2(unpack2<T>(v.x)) || !finite2(unpack2<T>(v.y)) || !finite2(unpack2<T>(v.z)) ||
            !finite2(unpack2<T>(v.w)))
          st |= NSNKV_ST_INPUT_NONFINITE;
      }
      *reinterpret_cast<uint4 *>(&S.qtile[c8 * 64 + r * 8]) = v;
    }
    fence_async_smem();
  }
  tc_fence_before();
  __syncthreads();  // barriers initialised, TMEM address and q tile visible
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;

  if (warp < kRestoreWarps) {
    // ---------------- restore: channel group cg of tokens 32*th..32*th+31 (lane = token)
    const int cg = warp & 3, th = warp >> 2, t = 32 * th + lane, mi = meta_index(32 * cg);
    const bool can_store = tl < a.tsh;
    if (is_raw && a.knew && !can_store && tl >= raw0 && tl < raw1 && tid == 0) st |= NSNKV_ST_CAPACITY;
    for (int u = 0; u < units; ++u) {
      const bool isv = u >= n;
      const int ui = isv ? u - n : u;
      const int s = u % kStages;
      if (!is_raw && !__all_sync(0xffffffffu, tc_wait(&S.ready[s], (u / kStages) & 1, a.status, abort))) break;
      if (u >= 2 && !__all_sync(0xffffffffu, tc_wait(&S.tempty[u & 1], ((u >> 1) - 1) & 1, a.status, abort))) break;
      uint32_t row[16];
      if (!is_raw) {
        const Stage<BITS> &sg = S.stage[s];
        float2 d[16];
        S.ssp[u & 1][cg][t] = restore_part<BITS>(sg.codes, sg.fa, sg.fb, mi, t, cg, d);
        // the four channel groups of this token half exchange their partial sums
        asm volatile("bar.sync %0, 128;" ::"r"(2 + th) : "memory");
        const float ss = (S.ssp[u & 1][0][t] + S.ssp[u & 1][1][t]) + (S.ssp[u & 1][2][t] + S.ssp[u & 1][3][t]);
        restore_finish<T>(d, renorm(half_bits_to_f(sg.norm[t]), ss), row);
      } else {
        const int j = raw0 + ui * kBlock + t;
        const T *base = static_cast<const T *>(isv ? a.vt : a.kt) + (b * a.tss + h * a.tsh) * kDim;
        const void *fresh_v = isv ? a.vnew : a.knew;
        const T *fresh = fresh_v ? static_cast<const T *>(fresh_v) + (b * a.h + h) * kDim : nullptr;
        if (j < raw1) {
          const bool is_new = fresh && j == tl;
          load_row32<T>(is_new ? fresh : base + static_cast<int64_t>(j) * kDim, 32 * cg, row);
          st |= check_row32<T>(row);
          // the appended token is written into the tail buffer at index tl
          if (is_new && can_store)
            store_row32(reinterpret_cast<uint16_t *>(const_cast<T *>(base) + static_cast<int64_t>(j) * kDim) + 32 * cg,
                        row);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) row[i] = 0u;
        }
      }
      uint16_t *tile = S.tile[u & 1];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int c8 = 4 * cg + jj;
        const int off = isv ? c8 * 512 + (t >> 3) * 64 + (t & 7) * 8 : (t >> 3) * 1024 + c8 * 64 + (t & 7) * 8;
        *reinterpret_cast<uint4 *>(tile + off) = make_uint4(row[4 * jj], row[4 * jj + 1], row[4 * jj + 2], row[4 * jj + 3]);
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&S.tfull[u & 1]);
        if (!is_raw) mbar_arrive(&S.empty[s]);
      }
    }
    // ---------------- epilogue: warps 0..3 read the P.V accumulator of channels 32w..32w+31
    if (warp < 4 && __all_sync(0xffffffffu, tc_wait(&S.d2full, 0, a.status, abort))) {
      tc_fence_after();
      uint32_t r[16];
      tmem_ld16(tmem + (static_cast<uint32_t>(32 * warp) << 16) + 16u, r);
      tmem_wait_ld();
      const int c = 32 * warp + lane;
#pragma unroll
      for (int gg = 0; gg < kHeads; ++gg) {
        if (gg < G) {
          const int64_t prow = (b * a.hq + h * G + gg) * a.max_chunks + chunk;
          a.part_o[prow * kDim + c] = __uint_as_float(r[gg]) + __uint_as_float(r[kHeads + gg]);
        }
      }
    }
  } else if (warp >= kSoftmaxWarp0 && warp < kSoftmaxWarp0 + kSoftmaxWarps) {
    // ---------------- softmax: K phase (scores, exact chunk maximum) then V phase (P).
    // Lane l < 16 of warp 8+q owns token 16q + l of every unit.
    const int q = warp - kSoftmaxWarp0, t = 16 * q + (lane & 15);
    const bool act = lane < 16;
    const uint32_t tq = tmem + (static_cast<uint32_t>(32 * q) << 16);
    float m[kHeads];
#pragma unroll
    for (int g = 0; g < kHeads; ++g) m[g] = -INFINITY;
    bool ok = true;
    for (int u = 0; u < n; ++u) {
      ok = __all_sync(0xffffffffu, tc_wait(&S.d1full[u & 1], (u >> 1) & 1, a.status, abort));
      if (!ok) break;
      tc_fence_after();
      uint32_t r[8];
      tmem_ld8(tq + 8u * (u & 1), r);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.d1empty[u & 1]);
      const int valid = is_raw ? min(kBlock, raw1 - (raw0 + u * kBlock)) : kBlock;
      if (act) {
#pragma unroll
        for (int g = 0; g < kHeads; ++g) {
          const float sc = t < valid ? __uint_as_float(r[g]) * kScale : -INFINITY;
          m[g] = fmaxf(m[g], sc);
          S.scores[g][u * kBlock + t] = sc;
        }
      }
    }
    // chunk maximum of each head: over the 16 lanes, then over the four warps
#pragma unroll
    for (int g = 0; g < kHeads; ++g) {
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) m[g] = fmaxf(m[g], __shfl_xor_sync(0xffffffffu, m[g], o));
    }
    if (lane == 0) {
#pragma unroll
      for (int g = 0; g < kHeads; ++g) S.red[q][g] = m[g];
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kSoftmaxWarps * 32) : "memory");
    float mb[kHeads];
#pragma unroll
    for (int g = 0; g < kHeads; ++g) {
      m[g] = fmaxf(fmaxf(S.red[0][g], S.red[1][g]), fmaxf(S.red[2][g], S.red[3][g]));
      mb[g] = m[g] * kLog2e;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kSoftmaxWarps * 32) : "memory");  // S.red is reused for the sums
    float l[kHeads];
#pragma unroll
    for (int g = 0; g < kHeads; ++g) l[g] = 0.f;
    for (int v = 0; v < n && ok; ++v) {
      const int pb = v & 1;
      if (v >= 2) {
        ok = __all_sync(0xffffffffu, tc_wait(&S.pempty[pb], ((v >> 1) - 1) & 1, a.status, abort));
        if (!ok) break;
      }
      if (act) {
        float p[kHeads];
#pragma unroll
        for (int g = 0; g < kHeads; ++g) {
          const float sc = S.scores[g][v * kBlock + t];
          p[g] = (g < G && m[g] != -INFINITY) ? exp2f(fmaf(sc, kLog2e, -mb[g])) : 0.f;
          l[g] += p[g];
        }
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          hi[i] = pack2<T>(f2(p[2 * i], p[2 * i + 1]));
          const float2 hv = unpack2<T>(hi[i]);
          lo[i] = pack2<T>(f2(p[2 * i] - hv.x, p[2 * i + 1] - hv.y));
        }
        uint16_t *pt = S.ptile[pb] + (t >> 3) * 64 + (t & 7) * 8;
        *reinterpret_cast<uint4 *>(pt) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4 *>(pt + 512) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.pfull[pb]);
    }
#pragma unroll
    for (int g = 0; g < kHeads; ++g) {
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) l[g] += __shfl_xor_sync(0xffffffffu, l[g], o);
    }
    if (lane == 0) {
#pragma unroll
      for (int g = 0; g < kHeads; ++g) S.red[q][g] = l[g];
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kSoftmaxWarps * 32) : "memory");
    if (ok && q == 0 && lane < G) {
      float lm = 0.f, ls = 0.f;
#pragma unroll
      for (int g = 0; g < kHeads; ++g) {
        if (g == lane) {
          lm = m[g];
          ls = (S.red[0][g] + S.red[1][g]) + (S.red[2][g] + S.red[3][g]);
        }
      }
      const int64_t prow = (b * a.hq + h * G + lane) * a.max_chunks + chunk;
      a.part_ml[prow * 2] = lm;
      a.part_ml[prow * 2 + 1] = ls;
    }
  } else if (warp == kProducerWarp) {
    // ---------------- producer: TMA ring and restore coefficients (sealed chunks)
    if (!is_raw) {
      const float fac = static_cast<float>(1 << (23 - code_pos<BITS>(lane)));
      int issued = 0, landed = 0;
      auto issue = [&](int u) {
        const int s = u % kStages;
        const bool isv = u >= n;
        const int i = blk0 + (isv ? u - n : u);
        const int32_t page = a.table ? a.table[b * a.table_stride + i] : i;
        const int64_t bi = static_cast<int64_t>(h) * a.sh + static_cast<int64_t>(page) * a.sp;
        Stage<BITS> &sg = S.stage[s];
        if (lane == 0) {
          mbar_expect_tx(&S.full[s], CB + kBlock * 2 + 2 * kDim * 2);
          bulk_g2s(sg.codes, (isv ? a.vc : a.kc) + bi * CB, CB, &S.full[s]);
          bulk_g2s(sg.norm, (isv ? a.vn : a.kn) + bi * kBlock, kBlock * 2, &S.full[s]);
          bulk_g2s(sg.mn, (isv ? a.vm : a.km) + bi * kDim, kDim * 2, &S.full[s]);
          bulk_g2s(sg.sc, (isv ? a.vs : a.ks) + bi * kDim, kDim * 2, &S.full[s]);
        }
        ++issued;
      };
      for (int u = 0; u < units && u < kStages; ++u) issue(u);
      for (int u = 0; u < units; ++u) {
        const int s = u % kStages;
        if (!__all_sync(0xffffffffu, tc_wait(&S.full[s], (u / kStages) & 1, a.status, abort))) break;
        ++landed;
        Stage<BITS> &sg = S.stage[s];
        bool bad = false;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c = lane + 32 * i, ci = meta_index(c);
          const float m = half_bits_to_f(sg.mn[c]), sc = half_bits_to_f(sg.sc[c]);
          const float bb = sc * fac;
          sg.fa[ci] = m - bb;
          sg.fb[ci] = bb;
          bad |= !isfinite(m) || !isfinite(sc);
        }
        bad |= !isfinite(half_bits_to_f(sg.norm[lane])) || !isfinite(half_bits_to_f(sg.norm[lane + 32]));
        if (bad) st |= NSNKV_ST_INPUT_NONFINITE;
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.ready[s]);
        const int nx = u - 1 + kStages;
        if (u >= 1 && nx < units) {
          if (!__all_sync(0xffffffffu, tc_wait(&S.empty[(u - 1) % kStages], ((u - 1) / kStages) & 1, a.status, abort)))
            break;
          issue(nx);
        }
      }
      // copies still in flight after an abort: a bounded wait each before the CTA leaves
      for (int u = landed; u < issued; ++u) mbar_wait_bounded(&S.full[u % kStages], (u / kStages) & 1, a.status);
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issue (one thread)
    if (lane == 0) {
      constexpr uint32_t kIdQK = umma_idesc<T>(kBlock, kHeads, 0, 0);
      constexpr uint32_t kIdPV = umma_idesc<T>(128, 16, 1, 1);
      const uint32_t qa = smem_addr(S.qtile);
      for (int u = 0; u < units; ++u) {
        const int buf = u & 1;
        if (!tc_wait(&S.tfull[buf], (u >> 1) & 1, a.status, abort)) break;
        tc_fence_after();
        const uint32_t ta = smem_addr(S.tile[buf]);
        if (u < n) {
          if (u >= 2) {
            if (!tc_wait(&S.d1empty[buf], ((u >> 1) - 1) & 1, a.status, abort)) break;
            tc_fence_after();
          }
#pragma unroll
          for (int k = 0; k < kDim / 16; ++k)
            umma_f16(tmem + 8u * buf, umma_desc(ta + 256u * k, 128u, 2048u), umma_desc(qa + 256u * k, 128u, 1024u),
                     kIdQK, k);
          umma_commit(&S.tempty[buf]);
          umma_commit(&S.d1full[buf]);
        } else {
          const int v = u - n, pb = v & 1;
          if (!tc_wait(&S.pfull[pb], (v >> 1) & 1, a.status, abort)) break;
          tc_fence_after();
          const uint32_t pa = smem_addr(S.ptile[pb]);
#pragma unroll
          for (int k = 0; k < kBlock / 16; ++k)
            umma_f16(tmem + 16u, umma_desc(ta + 256u * k, 128u, 1024u), umma_desc(pa + 256u * k, 128u, 1024u), kIdPV,
                     (v > 0 || k > 0) ? 1u : 0u);
          umma_commit(&S.tempty[buf]);
          umma_commit(&S.pempty[pb]);
          if (v == n - 1) umma_commit(&S.d2full);
        }
      }
      // every MMA issued has completed before TMEM is released
      umma_commit(&S.done);
      mbar_wait_bounded(&S.done, 0, a.status);
    }
    __syncwarp();
  }

  if (st) set_status(a.status, st);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// Combine the chunk partials of one (sequence, query head).
template <typename T>
__global__ void __launch_bounds__(128) attn_merge_kernel(const AttnArgs a, int G, T *out, float *out_f32,
                                                          float *lse) {
  const int hqi = blockIdx.x;
  const int64_t b = blockIdx.y;
  const int c = threadIdx.x;
  const int nb = a.nblk ? a.nblk[b] : a.nblk_const;
  const int tl = a.tlen ? a.tlen[b] : a.tlen_const;
  const int tail_total = tl + (a.knew ? 1 : 0);
  const int raw_per_chunk = a.chunk_blocks * kBlock;
  const int n_chunks = (nb + a.chunk_blocks - 1) / a.chunk_blocks + (tail_total + raw_per_chunk - 1) / raw_per_chunk;
  const int64_t row0 = (b * a.hq + hqi) * a.max_chunks;
  float M = -INFINITY;
  for (int i = 0; i < n_chunks; ++i) M = fmaxf(M, a.part_ml[(row0 + i) * 2]);
  float L = 0.f, o = 0.f;
  constexpr float kLog2e = 1.4426950408889634f;
  for (int i = 0; i < n_chunks; ++i) {
    const float m = a.part_ml[(row0 + i) * 2];
    const float w = m == -INFINITY ? 0.f : exp2f((m - M) * kLog2e);
    L += w * a.part_ml[(row0 + i) * 2 + 1];
    o += w * a.part_o[(row0 + i) * kDim + c];
  }
  const float y = __fdiv_rn(o, L);
  const T yt = Elem<T>::from_f(y);
  const int64_t orow = b * a.hq + hqi;
  out[orow * kDim + c] = yt;
  if (out_f32) out_f32[orow * kDim + c] = y;
  if (lse && c == 0) lse[orow] = M + logf(L);
  if (!isfinite(Elem<T>::to_f(yt)) || !isfinite(y)) set_status(a.status, NSNKV_ST_OUTPUT_NONFINITE);
}

// Combine per-shard (o, lse) rows: used after an all-gather in the split-KV path.
template <typename T>
__global__ void __launch_bounds__(128) merge_shards_kernel(int n_shards, int64_t rows, const float *o,
                                                            const float *lse_in, T *out, float *out_f32,
                                                            float *lse_out, int32_t *status) {
  const int64_t r = blockIdx.x;
  const int c = threadIdx.x;
  float M = -INFINITY;
  for (int s = 0; s < n_shards; ++s) M = fmaxf(M, lse_in[s * rows + r]);
  float L = 0.f, acc = 0.f;
  for (int s = 0; s < n_shards; ++s) {
    const float l = lse_in[s * rows + r];
    const float w = l == -INFINITY ? 0.f : expf(l - M);
    L += w;
    acc += w * o[(s * rows + r) * kDim + c];
  }
  const float y = __fdiv_rn(acc, L);
  const T yt = Elem<T>::from_f(y);
  out[r * kDim + c] = yt;
  if (out_f32) out_f32[r * kDim + c] = y;
  if (lse_out && c == 0) lse_out[r] = M + logf(L);
  if (!isfinite(Elem<T>::to_f(yt))) set_status(status, NSNKV_ST_OUTPUT_NONFINITE);
}

// ----------------------------------------------------------------- host side
static int chunk_blocks_for(int64_t batch, int h, int32_t max_blocks, int32_t max_tail) {
  // Aim for >= 4 CTAs per SM (148 SMs) while keeping the partials small.
  const int64_t units = batch * h;
  const int64_t target = 148 * 12;
  const int64_t work = max_blocks + (static_cast<int64_t>(max_tail) + 1 + kBlock - 1) / kBlock;
  int64_t per_unit = (target + units - 1) / units;  // desired chunks per (seq, head)
  int64_t ch = (work + per_unit - 1) / per_unit;
  if (ch < 4) ch = 4;
  if (ch > kChunk) ch = kChunk;
  return static_cast<int>(ch);
}

static int max_chunks_for(int32_t max_blocks, int32_t max_tail, int32_t ch) {
  const int64_t raw = static_cast<int64_t>(max_tail) + 1;  // +1: an appended token
  return static_cast<int>((max_blocks + ch - 1) / ch + (raw + static_cast<int64_t>(ch) * kBlock - 1) / (static_cast<int64_t>(ch) * kBlock));
}

template <int BITS, typename T>
static int launch_attn(const AttnArgs &a, dim3 grid, cudaStream_t st) {
  auto k = attn_partial_kernel<BITS, T>;
  const size_t smem = sizeof(AttnSmem<BITS>);
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return NSNKV_ERR_CUDA;
  k<<<grid, kThreads, smem, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? NSNKV_OK : NSNKV_ERR_LAUNCH;
}

template <typename T>
static int dispatch_bits(int bits, int G, const AttnArgs &a, dim3 grid, cudaStream_t st) {
  if (G < 1 || G > kHeads) return NSNKV_ERR_UNSUPPORTED;
  switch (bits) {
    case 3: return launch_attn<3, T>(a, grid, st);
    case 4: return launch_attn<4, T>(a, grid, st);
    case 5: return launch_attn<5, T>(a, grid, st);
    default: return NSNKV_ERR_ARG;
  }
}

}  // namespace nsnkv

using namespace nsnkv;

extern "C" {

int64_t nsnkv_decode_attn_workspace_bytes(int64_t batch, int hq, int h, int32_t max_blocks, int32_t max_tail) {
  if (batch <= 0 || hq <= 0 || h <= 0 || max_blocks < 0) return 0;
  if (max_tail < 0) return 0;
  const int ch = chunk_blocks_for(batch, h, max_blocks, max_tail);
  const int64_t mc = max_chunks_for(max_blocks, max_tail, ch);
  return batch * hq * mc * (kDim + 2) * static_cast<int64_t>(sizeof(float));
}

int nsnkv_decode_attn(int64_t batch, int hq, int h, int bits, int dtype, const void *q, const uint8_t *k_codes,
                      const uint16_t *k_norm, const uint16_t *k_min, const uint16_t *k_scale, const uint8_t *v_codes,
                      const uint16_t *v_norm, const uint16_t *v_min, const uint16_t *v_scale, int64_t blk_stride_head,
                      int64_t blk_stride_page, const int32_t *block_table, int64_t table_stride,
                      const int32_t *n_blocks, int32_t n_blocks_const, int32_t max_blocks, void *k_tail, void *v_tail,
                      int64_t tail_stride_seq, int64_t tail_stride_head, const int32_t *tail_len,
                      int32_t tail_len_const, int32_t max_tail, const void *k_new, const void *v_new, void *out,
                      float *out_f32, float *lse, void *workspace, int64_t workspace_bytes, int32_t *status,
                      void *stream) {
  if (batch <= 0 || hq <= 0 || h <= 0 || hq % h != 0 || max_blocks < 0 || max_tail < 0) return NSNKV_ERR_ARG;
  if (bits < 3 || bits > 5 || (dtype != NSNKV_F16 && dtype != NSNKV_BF16)) return NSNKV_ERR_ARG;
  if (!q || !out || !status || !workspace || !aligned16(q) || !aligned16(out)) return NSNKV_ERR_ARG;
  if ((k_new == nullptr) != (v_new == nullptr)) return NSNKV_ERR_ARG;
  if (max_blocks > 0) {
    if (!k_codes || !k_norm || !k_min || !k_scale || !v_codes || !v_norm || !v_min || !v_scale) return NSNKV_ERR_ARG;
    const void *ptrs[] = {k_codes, k_norm, k_min, k_scale, v_codes, v_norm, v_min, v_scale};
    for (const void *p : ptrs)
      if (!aligned16(p)) return NSNKV_ERR_ARG;
  }
  const bool any_tail = max_tail > 0 || k_new != nullptr;
  if (any_tail && (!k_tail || !v_tail || !aligned16(k_tail) || !aligned16(v_tail))) return NSNKV_ERR_ARG;
  if (k_new && (!aligned16(k_new) || !aligned16(v_new))) return NSNKV_ERR_ARG;
  if (!n_blocks && n_blocks_const > max_blocks) return NSNKV_ERR_ARG;
  if (!tail_len && tail_len_const > max_tail) return NSNKV_ERR_ARG;
  if (workspace_bytes < nsnkv_decode_attn_workspace_bytes(batch, hq, h, max_blocks, max_tail)) return NSNKV_ERR_ARG;
  if (batch > 65535 || h > 65535) return NSNKV_ERR_ARG;

  AttnArgs a{};
  a.batch = batch;
  a.hq = hq;
  a.h = h;
  a.q = q;
  a.kc = k_codes;
  a.kn = k_norm;
  a.km = k_min;
  a.ks = k_scale;
  a.vc = v_codes;
  a.vn = v_norm;
  a.vm = v_min;
  a.vs = v_scale;
  a.sh = blk_stride_head;
  a.sp = blk_stride_page;
  a.table = block_table;
  a.table_stride = table_stride;
  a.nblk = n_blocks;
  a.nblk_const = n_blocks_const;
  a.kt = k_tail;
  a.vt = v_tail;
  a.tss = tail_stride_seq;
  a.tsh = tail_stride_head;
  a.tlen = tail_len;
  a.tlen_const = tail_len_const;
  a.knew = k_new;
  a.vnew = v_new;
  a.chunk_blocks = chunk_blocks_for(batch, h, max_blocks, max_tail);
  a.max_chunks = max_chunks_for(max_blocks, max_tail, a.chunk_blocks);
  float *ws = static_cast<float *>(workspace);
  a.part_o = ws;
  a.part_ml = ws + batch * hq * static_cast<int64_t>(a.max_chunks) * kDim;
  a.status = status;
  const int G = hq / h;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dim3 grid(a.max_chunks, h, static_cast<unsigned>(batch));
  int rc = dtype == NSNKV_F16 ? dispatch_bits<__half>(bits, G, a, grid, st)
                              : dispatch_bits<__nv_bfloat16>(bits, G, a, grid, st);
  if (rc != NSNKV_OK) return rc;
  dim3 mgrid(hq, static_cast<unsigned>(batch));
  if (dtype == NSNKV_F16)
    attn_merge_kernel<__half><<<mgrid, kDim, 0, st>>>(a, G, static_cast<__half *>(out), out_f32, lse);
  else
    attn_merge_kernel<__nv_bfloat16><<<mgrid, kDim, 0, st>>>(a, G, static_cast<__nv_bfloat16 *>(out), out_f32, lse);
  return cudaGetLastError() == cudaSuccess ? NSNKV_OK : NSNKV_ERR_LAUNCH;
}

int nsnkv_merge_shards(int n_shards, int64_t rows, const float *o, const float *lse, int dtype, void *out,
                       float *out_f32, float *lse_out, int32_t *status, void *stream) {
  if (n_shards <= 0 || rows <= 0 || rows > 0x7FFFFFFF || !o || !lse || !out || !status) return NSNKV_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == NSNKV_F16)
    merge_shards_kernel<__half><<<static_cast<unsigned>(rows), kDim, 0, st>>>(n_shards, rows, o, lse,
                                                                            static_cast<__half *>(out), out_f32,
                                                                            lse_out, status);
  else if (dtype == NSNKV_BF16)
    merge_shards_kernel<__nv_bfloat16><<<static_cast<unsigned>(rows), kDim, 0, st>>>(
        n_shards, rows, o, lse, static_cast<__nv_bfloat16 *>(out), out_f32, lse_out, status);
  else
    return NSNKV_ERR_ARG;
  return cudaGetLastError() == cudaSuccess ? NSNKV_OK : NSNKV_ERR_LAUNCH;
}

}  // extern "C"

// ----------------------------------------------------------------- allocation-free variant
// Scratch for nsnkv_decode_attn_noalloc: the split-KV partials live in this fixed,
// file-scope device array instead of a caller-provided workspace.  Every GPU that
// loads the library holds NSNKV_NOALLOC_SCRATCH_BYTES of it until the process exits.
// In host code `g_noalloc_scratch` is only a host-side stand-in for the symbol, not a
// device address; the device address is obtained once per device below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[NSNKV_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void *g_scratch_address[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device, looked up on the first
// call for that device (with that device current) and cached afterwards.
int noalloc_scratch(void **out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return NSNKV_ERR_CUDA;
  if (dev >= kMaxDevices) return NSNKV_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_address[dev]) {
    void *ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) return NSNKV_ERR_CUDA;
    g_scratch_address[dev] = ptr;
  }
  *out = g_scratch_address[dev];
  return NSNKV_OK;
}
}  // namespace

extern "C" int nsnkv_decode_attn_noalloc(
    int64_t batch, int hq, int h, int bits, int dtype, const void *q, const uint8_t *k_codes, const uint16_t *k_norm,
    const uint16_t *k_min, const uint16_t *k_scale, const uint8_t *v_codes, const uint16_t *v_norm,
    const uint16_t *v_min, const uint16_t *v_scale, int64_t blk_stride_head, int64_t blk_stride_page,
    const int32_t *block_table, int64_t table_stride, const int32_t *n_blocks, int32_t n_blocks_const,
    int32_t max_blocks, void *k_tail, void *v_tail, int64_t tail_stride_seq, int64_t tail_stride_head,
    const int32_t *tail_len, int32_t tail_len_const, int32_t max_tail, const void *k_new, const void *v_new,
    void *out, float *out_f32, float *lse, int32_t *status, void *stream) {
  const int64_t need = nsnkv_decode_attn_workspace_bytes(batch, hq, h, max_blocks, max_tail);
  if (need <= 0) return NSNKV_ERR_ARG;
  if (need > NSNKV_NOALLOC_SCRATCH_BYTES) return NSNKV_ERR_TOO_LARGE;
  void *scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != NSNKV_OK) return rc;
  // The partials need no clearing: every entry the merge reads is written earlier in
  // the same call.  Calls that overlap on the GPU share the array and race.
  return nsnkv_decode_attn(batch, hq, h, bits, dtype, q, k_codes, k_norm, k_min, k_scale, v_codes, v_norm, v_min,
                           v_scale, blk_stride_head, blk_stride_page, block_table, table_stride, n_blocks,
                           n_blocks_const, max_blocks, k_tail, v_tail, tail_stride_seq, tail_stride_head, tail_len,
                           tail_len_const, max_tail, k_new, v_new, out, out_f32, lse, scratch,
                           NSNKV_NOALLOC_SCRATCH_BYTES, status, stream);
}
