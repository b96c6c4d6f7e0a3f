// Fused packed-KV decode attention for sm_100a (split-KV, flash-decoding style).
//
// One CTA (4 warps) owns (chunk of sealed blocks | a chunk of native rows, kv head h,
// sequence b) and serves all G = hq/h query heads of that kv head, so every packed
// byte is read from HBM exactly once (the reference's NB06 _partial re-reads each kv
// block G times, experiments/nb06/source/loop_kv_nb06_kernel.py:54-114).
//
// Per 64-token block, staged in shared memory by the TMA engine (cp.async.bulk,
// double buffered, completion on mbarriers):
//   K phase  warp w takes tokens 16w..16w+15; lane (g, tig) unpacks tokens g and g+8,
//            channels 32*tig..32*tig+31 in registers: d = min + scale*code (fp32),
//            row norm over a 4-lane shuffle, k = (norm/max(||d||,eps)) * d rounded to
//            the bridge dtype (fp16/bf16) -- the value restore_group would store --
//            and the packed pairs are used directly as the A fragments of
//            mma.m16n8k16 against q (B fragments, 8 query-head columns) -> scores.
//   softmax  running max / sum per query head, 2 heads per warp.
//   V phase  V rows are restored and rounded the same way into a padded shared tile;
//            P.V runs as mma.m16n8k16 with A = V^T loaded by ldmatrix.trans and
//            B = P split into hi + lo halves (fp32-accurate weights); warp w owns
//            channels 32w..32w+31 of the accumulator.
// Native rows (the tail, an appended token, or fully materialised K/V) use the same
// code without the unpack.  A merge kernel combines chunk partials with a
// log-sum-exp reduction (the reference's merge, loop_kv_af01_kernel.py:70-84).
#include <atomic>
#include <mutex>

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
  const float *ka, *va;  // per-token renorm factors (sealed INT3 path), or null
  int64_t sh, sp;
  int64_t cs, ms;    // bytes from one block to the next: code arrays, min / scale / factor arrays
  int32_t one_copy;  // sealed kernel: each block's K then V arrays form one record of cs bytes
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
  int32_t raw_only;  // 1: CTA x takes the x-th native-row chunk (sealed chunks run in attn_sealed3_kernel)
  float *part_o;   // [batch][hq][max_chunks][128]
  float *part_ml;  // [batch][hq][max_chunks][2]
  int32_t *status;
  // fused merge (unit_finish): the last chunk CTA of a (sequence, kv head) merges its partials
  int32_t fused;
  uint32_t epoch;                // this call's arrival epoch (the host's call counter)
  unsigned long long *arrive;    // [batch][h] arrival words: epoch << 32 | chunks arrived
  void *out;                     // [batch][hq][128] of the call's dtype
  float *out_f32, *lse;          // may be null
};

constexpr int kThreads = 128;    // 4 warps; warp w owns tokens 16w..16w+15 of every block
constexpr int kWarps = kThreads / 32;
constexpr int kHeads = 8;        // MMA rows/columns for the query heads of one kv head (G <= 8)
constexpr int kVRow = kDim + 8;  // padded V tile row (272 B): ldmatrix rows hit distinct banks
constexpr int kStages = 4;       // TMA ring depth (blocks in flight per CTA)
constexpr int kMetaRow = kDim + kDim / 8;  // fp32 metadata row padded every 32 channels by 4 floats

template <int BITS>
struct Stage {
  uint8_t kc[code_bytes(BITS)];
  uint8_t vc[code_bytes(BITS)];
  uint16_t kn[kBlock];
  uint16_t km[kDim];
  uint16_t ks[kDim];
  uint16_t vn[kBlock];
  uint16_t vm[kDim];
  uint16_t vs[kDim];
};

// Per-block fp32 metadata in the form the restore uses.  A code k is dropped into
// mantissa bits [p, p+BITS) of 1.0f, giving x = 1 + k*2^(p-23); then
//   d = min + scale*k = b*x + a,   b = scale * 2^(23-p),   a = min - b.
struct MetaF {
  float ka[kMetaRow], kb[kMetaRow], va[kMetaRow], vb[kMetaRow];
};

struct MergeSmem {  // cross-warp combine at the end of a chunk (aliases the V tiles)
  float acc[kWarps][kHeads][kDim];
  float m[kWarps][kHeads];
  float l[kWarps][kHeads];
};

template <int BITS>
struct AttnSmem {
  Stage<BITS> stage[kStages];
  MetaF meta[2];
  union {
    uint16_t v16[kWarps][16][kVRow];  // each warp's restored V rows (bridge dtype)
    MergeSmem merge;
  } u;
  uint64_t full[kStages];
};

// Shared memory of a CTA that only handles native rows (the tensor-core path's tail grid):
// no TMA ring, so several such CTAs fit into the slot of one finished sealed CTA.
struct RawSmem {
  union {
    uint16_t v16[kWarps][16][kVRow];
    MergeSmem merge;
  } u;
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

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void *smem_row) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem_row));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

__device__ __forceinline__ bool finite2(float2 v) { return isfinite(v.x) && isfinite(v.y); }

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
  // x for codes 2m and 2m+1 (see MetaF).
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

// d for this lane's 32 channels of one row, plus the full-row sum of squares.
template <int BITS>
__device__ __forceinline__ float row_dirs(const RowCodes<BITS> &rc, const float *ma, const float *mb, int mi,
                                          float2 (&d)[16]) {
  float2 ss0 = f2(0.f, 0.f), ss1 = f2(0.f, 0.f);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 a4 = *reinterpret_cast<const float4 *>(&ma[mi + 4 * q]);
    const float4 b4 = *reinterpret_cast<const float4 *>(&mb[mi + 4 * q]);
    d[2 * q] = __ffma2_rn(f2(b4.x, b4.y), rc.xpair(2 * q), f2(a4.x, a4.y));
    d[2 * q + 1] = __ffma2_rn(f2(b4.z, b4.w), rc.xpair(2 * q + 1), f2(a4.z, a4.w));
    ss0 = __ffma2_rn(d[2 * q], d[2 * q], ss0);
    ss1 = __ffma2_rn(d[2 * q + 1], d[2 * q + 1], ss1);
  }
  float s = (ss0.x + ss1.x) + (ss0.y + ss1.y);
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  return s;
}

// Restore two rows (this lane's 32 channels of tokens t0 and t1) with their work
// interleaved, renormalise and round to the bridge dtype: out0/out1 pack channel pairs.
template <int BITS, typename T>
__device__ __forceinline__ void restore_two_rows(const uint8_t *codes, const float *ma, const float *mb, int mi,
                                                 int t0, int t1, int tig, float n0, float n1, uint32_t (&out0)[16],
                                                 uint32_t (&out1)[16]) {
  RowCodes<BITS> r0, r1;
  r0.load(codes, t0, tig);
  r1.load(codes, t1, tig);
  float2 d0[16], d1[16];
  float2 s0 = f2(0.f, 0.f), s1 = f2(0.f, 0.f);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 a4 = *reinterpret_cast<const float4 *>(&ma[mi + 4 * q]);
    const float4 b4 = *reinterpret_cast<const float4 *>(&mb[mi + 4 * q]);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int m = 2 * q + e;
      const float2 a2 = e ? f2(a4.z, a4.w) : f2(a4.x, a4.y);
      const float2 b2 = e ? f2(b4.z, b4.w) : f2(b4.x, b4.y);
      d0[m] = __ffma2_rn(b2, r0.xpair(m), a2);
      d1[m] = __ffma2_rn(b2, r1.xpair(m), a2);
      s0 = __ffma2_rn(d0[m], d0[m], s0);
      s1 = __ffma2_rn(d1[m], d1[m], s1);
    }
  }
  float ss0 = s0.x + s0.y, ss1 = s1.x + s1.y;
  ss0 += __shfl_xor_sync(0xffffffffu, ss0, 1);
  ss1 += __shfl_xor_sync(0xffffffffu, ss1, 1);
  ss0 += __shfl_xor_sync(0xffffffffu, ss0, 2);
  ss1 += __shfl_xor_sync(0xffffffffu, ss1, 2);
  const float al0 = n0 == 0.f ? 0.f : (ss0 > 1e-24f ? n0 * rsqrtf(ss0) : n0 * 1e12f);
  const float al1 = n1 == 0.f ? 0.f : (ss1 > 1e-24f ? n1 * rsqrtf(ss1) : n1 * 1e12f);
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    out0[m] = pack2<T>(__fmul2_rn(d0[m], f2(al0, al0)));
    out1[m] = pack2<T>(__fmul2_rn(d1[m], f2(al1, al1)));
  }
}

// norm / max(||d||, eps) from the row sum of squares (0 when the stored norm is 0).
__device__ __forceinline__ float renorm(float n, float ss) {
  return n == 0.f ? 0.f : (ss > 1e-24f ? n * rsqrtf(ss) : n * 1e12f);
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

// Round 32 floats (16 pairs) to the bridge dtype and store them as 64 contiguous bytes.
template <typename T>
__device__ __forceinline__ void store_pairs(uint16_t *dst, const float2 (&d)[16]) {
  uint4 *p = reinterpret_cast<uint4 *>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    p[i] = make_uint4(pack2<T>(d[4 * i]), pack2<T>(d[4 * i + 1]), pack2<T>(d[4 * i + 2]), pack2<T>(d[4 * i + 3]));
}

__device__ __forceinline__ void store_row32(uint16_t *dst, const uint32_t (&u)[16]) {
  uint4 *p = reinterpret_cast<uint4 *>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = make_uint4(u[4 * i], u[4 * i + 1], u[4 * i + 2], u[4 * i + 3]);
}

// Per-warp online softmax state and accumulator.  Lane (g, tig) owns query head g
// (m, l) and the accumulator of channels 16mt + {g, g+8}, heads 2tig, 2tig+1.
struct WarpState {
  float m = -INFINITY, l = 0.f;
  float acc[8][4];
};

// Scores of this warp's 16-token tile for query head g, from one K row (n-tile) at a
// time: s[0..1] = tokens {2tig, 2tig+1} (row t0 of each lane), s[2..3] = tokens
// {8+2tig, 9+2tig} (row t1).  D[head][token] = q . k over the 8 channel slices; A rows
// 8..15 are zero.
template <typename T>
__device__ __forceinline__ void qk_rows(const uint32_t (&aq)[16], const uint32_t (&k)[16], float (&s)[4]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) mma16816<T>(s, aq[2 * j], 0u, aq[2 * j + 1], 0u, k[2 * j], k[2 * j + 1]);
}

// Online softmax of one 16-token tile and the P.V update.  sc holds the raw scores
// (sc[0..1] tokens 2tig, 2tig+1; sc[2..3] tokens 8+2tig, 9+2tig; head g), v16 the tile's
// V rows in the bridge dtype; valid[i] masks token i.
template <typename T>
__device__ __forceinline__ void warp_softmax_pv(WarpState &ws, const float (&raw)[4], const uint16_t (*v16)[kVRow],
                                                const bool (&valid)[4], int G, int lane, int &st) {
  constexpr float kLog2e = 1.4426950408889634f;
  const int g = lane >> 2, tig = lane & 3;
  float sc[4];
  float bmax = -INFINITY;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    sc[i] = valid[i] ? raw[i] * kScale : -INFINITY;
    if (valid[i] && g < G && !isfinite(sc[i])) st |= NSNKV_ST_OUTPUT_NONFINITE;
    bmax = fmaxf(bmax, sc[i]);
  }
  bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 1));
  bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 2));
  const float mnew = fmaxf(ws.m, bmax);
  float r = 1.f, psum = 0.f, p[4];
  if (g < G && mnew != -INFINITY) {
    r = exp2f((ws.m - mnew) * kLog2e);
    const float mb = mnew * kLog2e;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      p[i] = exp2f(fmaf(sc[i], kLog2e, -mb));
      psum += p[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = 0.f;
  }
  psum += __shfl_xor_sync(0xffffffffu, psum, 1);
  psum += __shfl_xor_sync(0xffffffffu, psum, 2);
  ws.l = ws.l * r + psum;
  ws.m = mnew;
  // rescale the accumulator only when some head's running max moved in this warp
  if (!__all_sync(0xffffffffu, r == 1.f)) {
    const float r0 = __shfl_sync(0xffffffffu, r, 8 * tig), r1 = __shfl_sync(0xffffffffu, r, 8 * tig + 4);
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      ws.acc[mt][0] *= r0;
      ws.acc[mt][1] *= r1;
      ws.acc[mt][2] *= r0;
      ws.acc[mt][3] *= r1;
    }
  }
  // B fragments of P (tokens 2tig, 2tig+1 | 8+2tig, 9+2tig; column = head g), split into
  // hi + lo halves of the bridge dtype so the weights keep fp32 accuracy
  const uint32_t bh0 = pack2<T>(f2(p[0], p[1])), bh1 = pack2<T>(f2(p[2], p[3]));
  const float2 ha = unpack2<T>(bh0), hb = unpack2<T>(bh1);
  const uint32_t bl0 = pack2<T>(f2(p[0] - ha.x, p[1] - ha.y)), bl1 = pack2<T>(f2(p[2] - hb.x, p[3] - hb.y));
  const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    uint32_t a[4];
    ldmatrix_x4_trans(a, &v16[rr + 8 * (mi >> 1)][16 * mt + 8 * (mi & 1)]);
    mma16816<T>(ws.acc[mt], a[0], a[1], a[2], a[3], bh0, bh1);
    mma16816<T>(ws.acc[mt], a[0], a[1], a[2], a[3], bl0, bl1);
  }
}

// ----------------------------------------------------------------- fused merge
// With a.fused, every chunk CTA of a (sequence b, kv head h) unit counts itself in after
// writing its partial rows, and the CTA that completes the count merges the unit's rows:
// the log-sum-exp combine of the reference (experiments/ac08/source/loop_kv_af01_kernel.py:70-84)
// for the unit's G query heads, without a separate merge launch.  The count is a 64-bit
// word per unit, epoch << 32 | chunks arrived; a word holding another epoch (an earlier
// call, or uninitialised workspace) counts as zero, and the merging CTA leaves it at
// (epoch, 0), so CUDA-graph replays of one call also start from zero.  The CAS loop only
// retries when another CTA of the unit arrived in between, so it ends within the unit's
// chunk count; the iteration cap is a guard that reports NSNKV_ST_TIMEOUT.
constexpr int kFusedChunks = 32;  // longest chunk list a unit may have for the fused merge

__device__ __forceinline__ int unit_arrive(unsigned long long *word, uint32_t epoch, int32_t *status) {
  const unsigned long long base = static_cast<unsigned long long>(epoch) << 32;
  unsigned long long expect = base;  // the first arrival's guess
  for (int it = 0; it < (1 << 16); ++it) {
    const unsigned long long want = (expect >> 32) == epoch ? expect + 1ull : base + 1ull;
    const unsigned long long got = atomicCAS(word, expect, want);
    if (got == expect) return static_cast<int>(want & 0xffffffffull);
    expect = got;
  }
  set_status(status, NSNKV_ST_TIMEOUT);
  return -1;
}

// A unit without any token (no sealed block, no tail row) has no chunk CTA to merge it:
// the chunk-0 CTA, exiting early, writes what the merge of zero partials gives (0 / 0,
// flagged as a non-finite output).  Called by every thread of that CTA.
template <typename T>
__device__ void empty_unit(const AttnArgs &a, int64_t b, int h) {
  const int nb = a.nblk ? a.nblk[b] : a.nblk_const;
  const int tl = a.tlen ? a.tlen[b] : a.tlen_const;
  if (!a.fused || nb != 0 || tl + (a.knew ? 1 : 0) != 0) return;
  const int G = a.hq / a.h;
  const float y = __fdiv_rn(0.f, 0.f);
  for (int e = threadIdx.x; e < G * kDim; e += blockDim.x) {
    const int64_t orow = b * a.hq + static_cast<int64_t>(h) * G + e / kDim;
    static_cast<T *>(a.out)[orow * kDim + e % kDim] = Elem<T>::from_f(y);
    if (a.out_f32) a.out_f32[orow * kDim + e % kDim] = y;
    if (a.lse && e % kDim == 0) a.lse[orow] = -INFINITY;
  }
  if (threadIdx.x == 0) set_status(a.status, NSNKV_ST_OUTPUT_NONFINITE);
}

// Called by all kThreads threads of a chunk CTA after its partial rows are stored; sm is
// the CTA's dynamic shared memory, free at this point (>= 4 * kHeads * (kFusedChunks + 2) + 16 bytes).
// The merge keeps many loads in flight: warp w takes heads w, w + 4 with lane i on chunk i
// (weights and sums by shuffles), then each thread sums four channels of one head with
// 128-bit loads, eight chunks per round.
template <typename T>
__device__ void unit_finish(const AttnArgs &a, int64_t b, int h, uint8_t *sm) {
  static_assert(kFusedChunks == 32 && kThreads == 128, "one lane per chunk, four warps");
  if (!a.fused) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = a.hq / a.h;
  const int nb = a.nblk ? a.nblk[b] : a.nblk_const;
  const int tl = a.tlen ? a.tlen[b] : a.tlen_const;
  const int tail_total = tl + (a.knew ? 1 : 0);
  const int raw_per_chunk = a.chunk_blocks * kBlock;
  const int n_chunks = (nb + a.chunk_blocks - 1) / a.chunk_blocks + (tail_total + raw_per_chunk - 1) / raw_per_chunk;
  float (*wt)[kFusedChunks] = reinterpret_cast<float (*)[kFusedChunks]>(sm);
  float *Ls = reinterpret_cast<float *>(sm) + kHeads * kFusedChunks;
  float *Ms = Ls + kHeads;
  int *last = reinterpret_cast<int *>(Ms + kHeads);
  unsigned long long *word = a.arrive + b * a.h + h;
  // Release: the barrier orders every thread's partial stores before thread 0's fence, and
  // the fence (cumulative) makes them visible device-wide before the count.  Acquire: the
  // fence after the last count orders the other CTAs' partials before this CTA's L2 reads.
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    *last = unit_arrive(word, a.epoch, a.status) == n_chunks;
    __threadfence();
  }
  __syncthreads();
  if (!*last) return;
  const int64_t row0 = (b * a.hq + static_cast<int64_t>(h) * G) * a.max_chunks;
  constexpr float kLog2e = 1.4426950408889634f;
  for (int n = warp; n < G; n += kWarps) {  // lane i: chunk i of head n
    float2 ml = make_float2(-INFINITY, 0.f);
    if (lane < n_chunks)
      ml = __ldcg(reinterpret_cast<const float2 *>(a.part_ml) + row0 + static_cast<int64_t>(n) * a.max_chunks + lane);
    float M = ml.x;
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float w = ml.x == -INFINITY ? 0.f : exp2f((ml.x - M) * kLog2e);  // no finite score: no weight
    float L = w * ml.y;
#pragma unroll
    for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    wt[n][lane] = w;
    if (lane == 0) {
      Ls[n] = L;
      Ms[n] = M;
    }
  }
  __syncthreads();
  int st = 0;
  for (int e = tid; e < G * (kDim / 4); e += kThreads) {
    const int n = e / (kDim / 4), c = 4 * (e % (kDim / 4));
    const float4 *po = reinterpret_cast<const float4 *>(a.part_o + (row0 + static_cast<int64_t>(n) * a.max_chunks) *
                                                                      kDim + c);
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int i = 0; i < n_chunks; ++i) {
      const float4 x = __ldcg(po + static_cast<int64_t>(i) * (kDim / 4));
      const float w = wt[n][i];
      o.x = fmaf(w, x.x, o.x);
      o.y = fmaf(w, x.y, o.y);
      o.z = fmaf(w, x.z, o.z);
      o.w = fmaf(w, x.w, o.w);
    }
    const float L = Ls[n];
    const float y[4] = {__fdiv_rn(o.x, L), __fdiv_rn(o.y, L), __fdiv_rn(o.z, L), __fdiv_rn(o.w, L)};
    const int64_t orow = b * a.hq + static_cast<int64_t>(h) * G + n;
    T *out = static_cast<T *>(a.out) + orow * kDim + c;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const T yt = Elem<T>::from_f(y[j]);
      out[j] = yt;
      if (!isfinite(Elem<T>::to_f(yt)) || !isfinite(y[j])) st = NSNKV_ST_OUTPUT_NONFINITE;
    }
    if (a.out_f32)  // (only 4-byte alignment is required of out_f32)
#pragma unroll
      for (int j = 0; j < 4; ++j) a.out_f32[orow * kDim + c + j] = y[j];
    if (a.lse && c == 0) a.lse[orow] = Ms[n] + logf(L);
  }
  if (st) set_status(a.status, st);
  if (tid == 0) atomicExch(word, static_cast<unsigned long long>(a.epoch) << 32);
}

// RAW: the CTA only ever takes native-row chunks (raw_only launches), with RawSmem.
template <int BITS, typename T, bool RAW = false>
__device__ __forceinline__ void attn_partial_cta(const AttnArgs &a, uint8_t *smem_raw) {
  constexpr int CB = code_bytes(BITS);
  using SmemT = typename std::conditional<RAW, RawSmem, AttnSmem<BITS>>::type;
  SmemT &S = *reinterpret_cast<SmemT *>(smem_raw);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tig = lane & 3, cbase = 32 * tig, mi = meta_index(cbase);
  const int t0 = 16 * warp + g, t1 = t0 + 8;
  const int h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int G = a.hq / a.h;

  const int nb = a.nblk ? a.nblk[b] : a.nblk_const;
  const int tl = a.tlen ? a.tlen[b] : a.tlen_const;
  const int tail_total = tl + (a.knew ? 1 : 0);
  const int n_sealed_chunks = (nb + a.chunk_blocks - 1) / a.chunk_blocks;
  const int raw_per_chunk = a.chunk_blocks * kBlock;
  const int n_chunks = n_sealed_chunks + (tail_total + raw_per_chunk - 1) / raw_per_chunk;
  const int chunk = a.raw_only ? n_sealed_chunks + static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x);
  if (chunk >= n_chunks) {
    if (blockIdx.x == 0) empty_unit<T>(a, b, h);
    return;
  }
  const bool is_raw = chunk >= n_sealed_chunks;

  int st = 0;
  // A fragments of q (rows = query heads h*G + g, zero when g >= G; rows 8..15 zero)
  uint32_t aq[16];
  if (g < G) {
    load_row32<T>(static_cast<const T *>(a.q) + ((b * a.hq) + h * G + g) * kDim, cbase, aq);
    st |= check_row32<T>(aq);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) aq[i] = 0u;
  }
  WarpState ws;
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) ws.acc[mt][0] = ws.acc[mt][1] = ws.acc[mt][2] = ws.acc[mt][3] = 0.f;
  uint16_t (*v16)[kVRow] = S.u.v16[warp];
  const bool all_valid[4] = {true, true, true, true};

  auto native_rows = [&]() {
    // ---- native rows (tail, appended token, or materialised K/V), per warp 16 rows of each 64-row tile
    const T *ktb = static_cast<const T *>(a.kt) + (b * a.tss + h * a.tsh) * kDim;
    const T *vtb = static_cast<const T *>(a.vt) + (b * a.tss + h * a.tsh) * kDim;
    const T *kn_row = a.knew ? static_cast<const T *>(a.knew) + (b * a.h + h) * kDim : nullptr;
    const T *vn_row = a.vnew ? static_cast<const T *>(a.vnew) + (b * a.h + h) * kDim : nullptr;
    const int raw0 = (chunk - n_sealed_chunks) * raw_per_chunk;
    const int raw1 = min(tail_total, raw0 + raw_per_chunk);
    const bool can_store = tl < a.tsh;
    if (a.knew && !can_store && tl >= raw0 && tl < raw1 && tid == 0) st |= NSNKV_ST_CAPACITY;
    const int ntiles = (raw1 - raw0 + kBlock - 1) / kBlock;
    for (int tile = 0; tile < ntiles; ++tile) {
      const int j0 = raw0 + tile * kBlock + t0, j1 = raw0 + tile * kBlock + t1;
      const bool v0 = j0 < raw1, v1 = j1 < raw1;
      auto row_ptr = [&](const T *base, const T *fresh_row, int j) -> const T * {
        return (fresh_row && j == tl) ? fresh_row : base + static_cast<int64_t>(j) * kDim;
      };
      uint32_t ka[16], kb[16], va[16], vb[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) ka[i] = kb[i] = va[i] = vb[i] = 0u;
      if (v0) {
        load_row32<T>(row_ptr(ktb, kn_row, j0), cbase, ka);
        load_row32<T>(row_ptr(vtb, vn_row, j0), cbase, va);
        st |= check_row32<T>(ka) | check_row32<T>(va);
      }
      if (v1) {
        load_row32<T>(row_ptr(ktb, kn_row, j1), cbase, kb);
        load_row32<T>(row_ptr(vtb, vn_row, j1), cbase, vb);
        st |= check_row32<T>(kb) | check_row32<T>(vb);
      }
      if (kn_row && can_store) {
        // the appended token is written into the tail buffers at index tl
        if (v0 && j0 == tl) {
          store_row32(reinterpret_cast<uint16_t *>(const_cast<T *>(ktb) + static_cast<int64_t>(j0) * kDim) + cbase, ka);
          store_row32(reinterpret_cast<uint16_t *>(const_cast<T *>(vtb) + static_cast<int64_t>(j0) * kDim) + cbase, va);
        }
        if (v1 && j1 == tl) {
          store_row32(reinterpret_cast<uint16_t *>(const_cast<T *>(ktb) + static_cast<int64_t>(j1) * kDim) + cbase, kb);
          store_row32(reinterpret_cast<uint16_t *>(const_cast<T *>(vtb) + static_cast<int64_t>(j1) * kDim) + cbase, vb);
        }
      }
      store_row32(&v16[g][cbase], va);
      store_row32(&v16[g + 8][cbase], vb);
      // validity of tokens 2tig, 2tig+1, 8+2tig, 9+2tig of this warp's 16 rows
      const int jb = raw0 + tile * kBlock + 16 * warp;
      const bool valid[4] = {jb + 2 * tig < raw1, jb + 2 * tig + 1 < raw1, jb + 8 + 2 * tig < raw1,
                             jb + 9 + 2 * tig < raw1};
      float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
      qk_rows<T>(aq, ka, s0);
      qk_rows<T>(aq, kb, s1);
      const float sraw[4] = {s0[0], s0[1], s1[0], s1[1]};
      __syncwarp();
      warp_softmax_pv<T>(ws, sraw, v16, valid, G, lane, st);
      __syncwarp();
    }
  
  };
  if constexpr (!RAW) {
    if (!is_raw) {
      const int blk0 = chunk * a.chunk_blocks;
      const int nloc = min(nb, blk0 + a.chunk_blocks) - blk0;
      auto issue = [&](int i, int s) {
        const int32_t page = a.table ? a.table[b * a.table_stride + i] : i;
        const int64_t bi = static_cast<int64_t>(h) * a.sh + static_cast<int64_t>(page) * a.sp;
        Stage<BITS> &sg = S.stage[s];
        mbar_expect_tx(&S.full[s], 2 * CB + 2 * (kBlock * 2 + 2 * kDim * 2));
        bulk_g2s(sg.kc, a.kc + bi * a.cs, CB, &S.full[s]);
        bulk_g2s(sg.vc, a.vc + bi * a.cs, CB, &S.full[s]);
        bulk_g2s(sg.kn, a.kn + bi * kBlock, kBlock * 2, &S.full[s]);
        bulk_g2s(sg.km, blk_ptr(a.km, bi, a.ms), kDim * 2, &S.full[s]);
        bulk_g2s(sg.ks, blk_ptr(a.ks, bi, a.ms), kDim * 2, &S.full[s]);
        bulk_g2s(sg.vn, a.vn + bi * kBlock, kBlock * 2, &S.full[s]);
        bulk_g2s(sg.vm, blk_ptr(a.vm, bi, a.ms), kDim * 2, &S.full[s]);
        bulk_g2s(sg.vs, blk_ptr(a.vs, bi, a.ms), kDim * 2, &S.full[s]);
      };
      if (tid == 0) {
#pragma unroll
        for (int i = 0; i < kStages; ++i) mbar_init(&S.full[i], 1);
        fence_mbar_init();
        for (int i = 0; i < kStages && i < nloc; ++i) issue(blk0 + i, i);
      }
      __syncthreads();  // no thread may poll a barrier before thread 0 has initialised it
      const float fac = static_cast<float>(1 << (23 - code_pos<BITS>(tid & 31)));
      for (int li = 0; li < nloc; ++li) {
        const int s = li % kStages;
        const bool ok = mbar_wait_bounded(&S.full[s], (li / kStages) & 1, a.status);
        const Stage<BITS> &sg = S.stage[s];
        MetaF &mf = S.meta[li & 1];
        if (ok) {  // fp32 metadata of this block, one channel per thread
          const int ci = meta_index(tid);
          const float km = half_bits_to_f(sg.km[tid]), ks = half_bits_to_f(sg.ks[tid]);
          const float vm = half_bits_to_f(sg.vm[tid]), vs = half_bits_to_f(sg.vs[tid]);
          const float kb_ = ks * fac, vb_ = vs * fac;
          mf.ka[ci] = km - kb_;
          mf.kb[ci] = kb_;
          mf.va[ci] = vm - vb_;
          mf.vb[ci] = vb_;
          bool bad = !isfinite(km) || !isfinite(ks) || !isfinite(vm) || !isfinite(vs);
          if (tid < kBlock) bad |= !isfinite(half_bits_to_f(sg.kn[tid])) || !isfinite(half_bits_to_f(sg.vn[tid]));
          if (bad) st |= NSNKV_ST_INPUT_NONFINITE;
        }
        if (__syncthreads_or(!ok)) {
          // A staged copy never landed: give the later copies a bounded chance to
          // finish, then leave; the timeout status tells the host.
          if (tid == 0)
            for (int k = li + 1; k < nloc && k < li + kStages; ++k)
              mbar_wait_bounded(&S.full[k % kStages], (k / kStages) & 1, a.status);
          return;
        }
        // every warp has finished block li-1: its stage takes block li-1+kStages
        if (tid == 0 && li >= 1 && li - 1 + kStages < nloc) issue(blk0 + li - 1 + kStages, (li - 1) % kStages);
        // ---- V rows t0, t1: restore, renormalise, round to the bridge dtype (the value
        // restore_group stores) into this warp's V tile
        {
          uint32_t u0[16], u1[16];
          restore_two_rows<BITS, T>(sg.vc, mf.va, mf.vb, mi, t0, t1, tig, half_bits_to_f(sg.vn[t0]),
                                    half_bits_to_f(sg.vn[t1]), u0, u1);
          store_row32(&v16[g][cbase], u0);
          store_row32(&v16[g + 8][cbase], u1);
        }
        // ---- K rows t0, t1: the same restore, then the scores of both rows
        float sraw[4];
        {
          uint32_t k0[16], k1[16];
          restore_two_rows<BITS, T>(sg.kc, mf.ka, mf.kb, mi, t0, t1, tig, half_bits_to_f(sg.kn[t0]),
                                    half_bits_to_f(sg.kn[t1]), k0, k1);
          // four independent accumulation chains per row (two slices each) shorten the
          // dependent MMA sequence; their sum is the score
          float s0[4][4], s1[4][4];
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < 4; ++i) s0[c][i] = s1[c][i] = 0.f;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            mma16816<T>(s0[j & 3], aq[2 * j], 0u, aq[2 * j + 1], 0u, k0[2 * j], k0[2 * j + 1]);
            mma16816<T>(s1[j & 3], aq[2 * j], 0u, aq[2 * j + 1], 0u, k1[2 * j], k1[2 * j + 1]);
          }
          sraw[0] = (s0[0][0] + s0[1][0]) + (s0[2][0] + s0[3][0]);
          sraw[1] = (s0[0][1] + s0[1][1]) + (s0[2][1] + s0[3][1]);
          sraw[2] = (s1[0][0] + s1[1][0]) + (s1[2][0] + s1[3][0]);
          sraw[3] = (s1[0][1] + s1[1][1]) + (s1[2][1] + s1[3][1]);
        }
        __syncwarp();
        warp_softmax_pv<T>(ws, sraw, v16, all_valid, G, lane, st);
        __syncwarp();
      }
    } else {
      native_rows();
    }
  } else {
    native_rows();
  }

  // ---- combine the four warps' partials and write this chunk's partial
  __syncthreads();
  MergeSmem &M = S.u.merge;
  if (tig == 0) {
    M.m[warp][g] = ws.m;
    M.l[warp][g] = ws.l;
  }
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    const int c = 16 * mt + g;
    M.acc[warp][2 * tig][c] = ws.acc[mt][0];
    M.acc[warp][2 * tig + 1][c] = ws.acc[mt][1];
    M.acc[warp][2 * tig][c + 8] = ws.acc[mt][2];
    M.acc[warp][2 * tig + 1][c + 8] = ws.acc[mt][3];
  }
  __syncthreads();
  constexpr float kLog2e = 1.4426950408889634f;
  for (int e = tid; e < G * kDim; e += kThreads) {
    const int n = e / kDim, c = e % kDim;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, M.m[w][n]);
    float o = 0.f, l = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float wt = M.m[w][n] == -INFINITY ? 0.f : exp2f((M.m[w][n] - mx) * kLog2e);
      o += wt * M.acc[w][n][c];
      l += wt * M.l[w][n];
    }
    const int64_t row = (b * a.hq + h * G + n) * a.max_chunks + chunk;
    a.part_o[row * kDim + c] = o;
    if (c == 0) {
      a.part_ml[row * 2] = mx;
      a.part_ml[row * 2 + 1] = l;
    }
  }
  if (st) set_status(a.status, st);
  unit_finish<T>(a, b, h, smem_raw);
}

// Programmatic dependent launch (sm_90+).  launch_dependents lets the next grid in the
// stream start once every CTA of this grid has issued it; wait returns once the grids
// this one depends on have completed and their memory is visible (at once when there
// are none).
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// The restore-path CTA (every shape without the tensor-core path, and the reference-layout
// entry points).  launch_dependents lets the merge grid, launched next with a programmatic
// dependency, become resident early; it waits for this grid on entry.  Launched normally,
// this grid has no programmatic predecessor, so its final wait returns at once.
template <int BITS, typename T>
__global__ void __launch_bounds__(kThreads, 3) attn_partial_kernel(const AttnArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  pdl_launch_dependents();  // the merge grid may be resident (and waiting) before this one ends
  attn_partial_cta<BITS, T>(a, smem_raw);
  pdl_wait();
}

// The tensor-core path's tail grid: the native-row chunks only (raw_only), with the small
// RawSmem.  Launched after attn_sealed3_kernel with a programmatic dependency, it fills
// slots freed in the sealed grid's last wave; the final wait keeps this grid from
// completing before the sealed grid, so the merge launched next sees both.
template <typename T>
__global__ void __launch_bounds__(kThreads, 4) attn_native_rows_kernel(const AttnArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  pdl_launch_dependents();
  attn_partial_cta<3, T, true>(a, smem_raw);
  pdl_wait();
}

// Combine the chunk partials of one (sequence, query head): the log-sum-exp merge of the
// reference (experiments/ac08/source/loop_kv_af01_kernel.py:70-84).  Thread c owns output
// channel c.  Up to kOnlineChunks chunks (batched decode) it walks them once, rescaling its
// running sum whenever a chunk raises the maximum: one round of independent loads and no
// block barrier.  Longer lists (one long sequence split into ~100 chunks) take two
// parallel passes instead: the chunks' (m, l) are read once by the CTA (thread i takes
// chunk i, i + 128, ...), their weights kept in shared memory, then every thread sums its
// channel with independent loads -- a serial online pass over that many chunks is a long
// dependent chain.
constexpr int kOnlineChunks = 16;
template <typename T>
__global__ void __launch_bounds__(128) attn_merge_kernel(const AttnArgs a, int G, T *out, float *out_f32,
                                                          float *lse) {
  pdl_wait();  // launched with a programmatic dependency: the partials are complete only now
  pdl_launch_dependents();
  const int hqi = blockIdx.x;
  const int64_t b = blockIdx.y;
  const int c = threadIdx.x;
  const int nb = a.nblk ? a.nblk[b] : a.nblk_const;
  const int tl = a.tlen ? a.tlen[b] : a.tlen_const;
  const int tail_total = tl + (a.knew ? 1 : 0);
  const int raw_per_chunk = a.chunk_blocks * kBlock;
  const int n_chunks = (nb + a.chunk_blocks - 1) / a.chunk_blocks + (tail_total + raw_per_chunk - 1) / raw_per_chunk;
  const int64_t row0 = (b * a.hq + hqi) * a.max_chunks;
  const float *ml = a.part_ml + row0 * 2;
  const float *po = a.part_o + row0 * kDim + c;
  constexpr float kLog2e = 1.4426950408889634f;
  float M = -INFINITY, L = 0.f, o = 0.f;
  if (n_chunks <= kOnlineChunks) {
#pragma unroll 4
    for (int i = 0; i < n_chunks; ++i) {
      const float m = ml[2 * i], l = ml[2 * i + 1], x = po[static_cast<int64_t>(i) * kDim];
      if (m == -INFINITY) continue;  // a chunk without a finite score contributes nothing
      if (m > M) {
        const float r = M == -INFINITY ? 0.f : exp2f((M - m) * kLog2e);
        L *= r;
        o *= r;
        M = m;
      }
      const float wgt = exp2f((m - M) * kLog2e);
      L = fmaf(wgt, l, L);
      o = fmaf(wgt, x, o);
    }
  } else {
    constexpr int kMaxW = 512;
    __shared__ float wgt[kMaxW];
    __shared__ float red[2][4];
    for (int i = c; i < n_chunks; i += kDim) M = fmaxf(M, ml[2 * i]);
#pragma unroll
    for (int s = 16; s; s >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, s));
    if ((c & 31) == 0) red[0][c >> 5] = M;
    __syncthreads();
    M = fmaxf(fmaxf(red[0][0], red[0][1]), fmaxf(red[0][2], red[0][3]));
    for (int i = c; i < n_chunks; i += kDim) {
      const float m = ml[2 * i];
      const float w = m == -INFINITY ? 0.f : exp2f((m - M) * kLog2e);
      L += w * ml[2 * i + 1];
      if (i < kMaxW) wgt[i] = w;
    }
#pragma unroll
    for (int s = 16; s; s >>= 1) L += __shfl_xor_sync(0xffffffffu, L, s);
    if ((c & 31) == 0) red[1][c >> 5] = L;
    __syncthreads();
    L = (red[1][0] + red[1][1]) + (red[1][2] + red[1][3]);
    if (n_chunks <= kMaxW) {
#pragma unroll 8
      for (int i = 0; i < n_chunks; ++i) o += wgt[i] * po[static_cast<int64_t>(i) * kDim];
    } else {
      for (int i = 0; i < n_chunks; ++i) {
        const float m = ml[2 * i];
        o += (m == -INFINITY ? 0.f : exp2f((m - M) * kLog2e)) * po[static_cast<int64_t>(i) * kDim];
      }
    }
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
// Shard s's rows start at o + s * o_stride and lse_in + s * lse_stride.
template <typename T>
__global__ void __launch_bounds__(128) merge_shards_kernel(int n_shards, int64_t rows, const float *o,
                                                            int64_t o_stride, const float *lse_in,
                                                            int64_t lse_stride, T *out, float *out_f32,
                                                            float *lse_out, int32_t *status) {
  const int64_t r = blockIdx.x;
  const int c = threadIdx.x;
  float M = -INFINITY;
  for (int s = 0; s < n_shards; ++s) M = fmaxf(M, lse_in[s * lse_stride + r]);
  float L = 0.f, acc = 0.f;
  for (int s = 0; s < n_shards; ++s) {
    const float l = lse_in[s * lse_stride + r];
    const float w = l == -INFINITY ? 0.f : expf(l - M);
    L += w;
    acc += w * o[s * o_stride + r * kDim + c];
  }
  const float y = __fdiv_rn(acc, L);
  const T yt = Elem<T>::from_f(y);
  out[r * kDim + c] = yt;
  if (out_f32) out_f32[r * kDim + c] = y;
  if (lse_out && c == 0) lse_out[r] = M + logf(L);
  if (!isfinite(Elem<T>::to_f(yt))) set_status(status, NSNKV_ST_OUTPUT_NONFINITE);
}

// ----------------------------------------------------------------- sealed INT3 blocks on the tensor cores
// attn_sealed3_kernel: the sealed chunks of INT3 fp16 caches with G <= 4 query heads per
// kv head, when per-token renorm factors alpha_t = n_t / max(||d_t||, eps) are stored
// beside the blocks (computed once at seal time by nsnkv_block_renorm).  With
// d = min + scale * code, a token's restored row is alpha_t * d, so
//   q . k_t = alpha_t * (sum_c q_c scale_c code_tc + sum_c q_c min_c)
//   sum_t p_t v_t = sum_t p_t alpha_t (min_c + scale_c code_tc)
// and both contractions take the 3-bit codes themselves as mma.sync operands.  One
// AND drops a code into the mantissa of an fp16 subnormal (value code * 2^(pos-24)),
// two codes per register; the per-channel scale goes into the other operand
// (K side: q * scale split exactly into fp16 hi + lo columns) or into an fp32
// epilogue per block (V side).  Each warp owns whole blocks: block li of the chunk
// goes to warp li % 4, which streams it through its own two-stage TMA ring and runs
//   K  4 m-tiles (16 tokens) x 9 k-steps of mma.m16n8k16: A = code pairs of a token,
//      B = [q_h * scale hi | lo] for the warp lane's head h = tig,
//   softmax over the block's 64 tokens for that head (running max / sum per warp),
//   V  8 m-tiles (16 channel slots) x 4 k-steps: A = code pairs of one channel in two
//      tokens, B = p * alpha split into hi | lo (movmatrix turns the score layout into
//      the B fragments), then acc += scale_c * D + min_c * sum_t p_t alpha_t.
// No restored K or V value is formed anywhere.
namespace s3 {

constexpr int kRing = 6;  // TMA stages per CTA: block li of a chunk lives in stage li % kRing
constexpr int kRec = 60;  // words of a lane's constant record: stride 4 * odd -> conflict-free 128-bit loads
constexpr int kCB = 3072;  // INT3 code bytes per block
constexpr int kMaxChunk = 32;  // blocks per chunk (page indices staged in shared memory)

// One block as the paged cache's block record holds it: K codes, min, scale, factors,
// then the same for V (one copy when the arrays are laid out so).
struct SStage {
  uint8_t kc[kCB];
  uint16_t km[kDim], ks[kDim];
  float ka[kBlock];
  uint8_t vc[kCB];
  uint16_t vm[kDim], vs[kDim];
  float va[kBlock];
};
static_assert(sizeof(SStage) == 7680 && offsetof(SStage, vc) == 3840, "stage layout = K record, V record");

struct SMerge {
  MergeSmem part;
  float wt[kWarps][kHeads];  // exp(m_warp - m_chunk) per (warp, head)
};

struct SSmem {
  union {
    SStage stage[kRing];
    SMerge merge;  // after the last block of every warp
  } u;
  uint32_t rec[32][kRec];  // per lane: [0,18) qa, [20,38) qz, [40,56) Delta A fragments
  __half qs[4][kDim];  // this kv head's query rows (G <= 4)
  int32_t pages[kMaxChunk];  // page of each block of the chunk
  // Block B completes on full[B % kRing][(B / kRing) & 1], parity (B / (2 kRing)) & 1.  Two
  // barriers per stage: warp B % 4 consumed block B - 2 kRing (the same barrier's previous
  // phase) before it waits for B, so a parity wait never meets a barrier two phases behind.
  uint64_t full[kRing][2];
  int32_t nissued[kRing][2];  // copies started per barrier (read only after a failed wait)
  int32_t failed;
};

// K side.  A lane group (tig) covers channels 32*tig + j, j = 0..31 of a token row: 96
// bits in three words w0..w2, code j at bits 3j..3j+2.  Source words X0..X5 are the
// group's bits starting at 0, 8, 32, 40, 64, 72; register r takes one code from the low
// 16 bits of X_src (start in [0, 8)) and one from the high 16 bits (start in [16, 24)),
// each staying below bit 10 of its half.  Columns: src, j_lo, pos_lo, j_hi, pos_hi
// (-1: the half stays zero).  18 registers = 9 k-steps of 16 channel slots.
__host__ __device__ constexpr int ktab(int r, int f) {
  constexpr int t[18][5] = {{0, 0, 0, 6, 2},    {0, 1, 3, 7, 5},    {0, 2, 6, -1, 0},  {1, 3, 1, 8, 0},
                            {1, 4, 4, 9, 3},    {1, 5, 7, 10, 6},   {2, 11, 1, 16, 0}, {2, 12, 4, 17, 3},
                            {2, 13, 7, 18, 6},  {3, 14, 2, 19, 1},  {3, 15, 5, 20, 4}, {3, -1, 0, 21, 7},
                            {4, 22, 2, 27, 1},  {4, 23, 5, 28, 4},  {4, -1, 0, 29, 7}, {5, 24, 0, 30, 2},
                            {5, 25, 3, 31, 5},  {5, 26, 6, -1, 0}};
  return t[r][f];
}
__host__ __device__ constexpr uint32_t kmask(int r) {
  return (ktab(r, 1) >= 0 ? 7u << ktab(r, 2) : 0u) | (ktab(r, 3) >= 0 ? 7u << (16 + ktab(r, 4)) : 0u);
}
// PRMT selector gathering the scales of register r's two channels from natural pairs.
__host__ __device__ constexpr uint32_t ksel(int r) {
  return (ktab(r, 1) >= 0 && (ktab(r, 1) & 1) ? 0x32u : 0x10u) |
         ((ktab(r, 3) >= 0 && (ktab(r, 3) & 1) ? 0x76u : 0x54u) << 8);
}

// V side.  Lane g covers channels 16g + i, i = 0..15: the 48-bit field F at bit 48g of
// a token row, code i at F bits 3i.  L = F bytes 0..3, H = F bytes 2..5; window k
// (0..5) is the 16-bit slice of F starting at byte k, taken from L (k < 3) or H, and
// a register holds channel i of two tokens: the window of each token in one half,
// then an AND at the code's position inside the window.
__host__ __device__ constexpr int vwin(int i) { return (3 * i) >> 3; }
__host__ __device__ constexpr int vpos(int i) { return 3 * i - 8 * vwin(i); }
__host__ __device__ constexpr uint32_t vsel(int k) {
  return k == 0 ? 0x5410u : (k == 1 || k == 3) ? 0x6521u : (k == 2 || k == 4) ? 0x7632u : 0x7733u;
}
// V operand of channel i (0..15 of a lane's field): codes at window positions 0..3 become
// normal fp16 code * 2^pos (OR 1024, subtract 1024: exact), the rest stay fp16 subnormals
// code * 2^(pos - 24).  Measured on B200: the P.V sums over the smallest subnormal operands
// lose precision in proportion to 2^-pos (about 2^-12 of the channel's value at position 0
// when one token carries most of the softmax weight); normal operands do not.  vunit(i) is
// the exponent of the operand's unit, so D and the per-channel accumulators count in 2^vunit.
constexpr int kVNormal = 3;  // highest window position given a normal operand
__host__ __device__ constexpr int vunit(int i) { return vpos(i) <= kVNormal ? vpos(i) : vpos(i) - 24; }

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) { return __byte_perm(a, b, sel); }

__device__ __forceinline__ uint32_t hsub2u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
constexpr uint32_t kMagic2 = 0x64006400u;  // fp16 1024 in both halves

// The V operand of channel i from window x (two tokens, one per half): see vunit.
__device__ __forceinline__ uint32_t vop(uint32_t x, int i) {
  const uint32_t c = x & (0x00070007u << vpos(i));
  return vpos(i) <= kVNormal ? hsub2u(c | kMagic2, kMagic2) : c;
}

__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hfma2u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// 2^x for x <= 0 (softmax weights): one MUFU.EX2; results below 2^-126 flush to zero.
__device__ __forceinline__ float ex2_neg(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t movtrans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
// An fp32 weight as fp16 hi (low half) and fp16 lo = RN(w - hi) (high half).
__device__ __forceinline__ uint32_t split_hilo(float w) {
  const float hf = __half2float(__float2half_rn(w));
  __half2 p = __floats2half2_rn(w, w - hf);
  return *reinterpret_cast<uint32_t *>(&p);
}

}  // namespace s3

// ----------------------------------------------------------------- the exact kernel's shared pieces
// The per-block arithmetic, the per-lane q records and the chunk combine of the exact
// sealed INT3 kernel (one CTA per chunk).  REC: the codes are in the paged cache's
// block-record orders (K paired halves, V paired rows); otherwise the reference's packed
// rows.
namespace s3 {

__device__ __forceinline__ float pow2f(int e) { return __int_as_float((127 + e) << 23); }  // 2^e, -126 <= e <= 127

// Per-lane constant records for the query rows qs (G <= 4 heads), the same in every warp:
// each of the four warps writes a quarter, so the caller synchronises the warps before any
// of them reads recs.  Returns kq of head tig (the exponent shift of its q columns).
template <bool REC>
__device__ __forceinline__ int build_records(const __half (*qs)[kDim], int G, uint32_t (*recs)[kRec], int lane,
                                             int warp) {
  const int g = lane >> 2, tig = lane & 3;
  auto pow2 = [](int e) { return pow2f(e); };
  // ---- per-head q exponent kq_h: |q_h| < 2^(8 + kq_h), so q * 2^(7 - pos - kq_h) is a finite fp16
  // (each MMA column is one head, so the shift may differ per head); every warp computes all four
  int kqh[4];
#pragma unroll
  for (int hh = 0; hh < 4; ++hh) {
    float mx = 0.f;
    if (hh < G) {
      const uint2 u = *reinterpret_cast<const uint2 *>(&qs[hh][4 * lane]);
      const float2 x0 = Elem<__half>::to_f2(u.x), x1 = Elem<__half>::to_f2(u.y);
      mx = fmaxf(fmaxf(fabsf(x0.x), fabsf(x0.y)), fmaxf(fabsf(x1.x), fabsf(x1.y)));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const int e = ((__float_as_int(mx) >> 23) & 0xff) - 126;  // mx < 2^e (frexp exponent)
    kqh[hh] = e > 8 ? e - 8 : 0;
  }
  auto pick = [&](int hh) { return hh == 0 ? kqh[0] : hh == 1 ? kqh[1] : hh == 2 ? kqh[2] : kqh[3]; };

  // ---- per-lane constant records (the same in every warp), each warp writing a quarter
  {
    uint32_t *rec = recs[lane];
    const int hb = g >> 1, pb = g & 1;
    const int kb = pick(hb);
#pragma unroll
    for (int r = 0; r < 18; ++r) {
      if ((r & 3) != warp) continue;
      float lo = 0.f, hi = 0.f;
      if (REC) {  // register r: channels 32 tig + r and 32 tig + 16 + r, both at window position vpos(r)
        if (r < 16 && hb < G) {
          lo = __half2float(qs[hb][32 * tig + r]) * pow2(7 - vpos(r) - kb);
          hi = __half2float(qs[hb][32 * tig + 16 + r]) * pow2(7 - vpos(r) - kb);
        }
      } else if (hb < G) {
        if (ktab(r, 1) >= 0) lo = __half2float(qs[hb][32 * tig + ktab(r, 1)]) * pow2(7 - ktab(r, 2) - kb);
        if (ktab(r, 3) >= 0) hi = __half2float(qs[hb][32 * tig + ktab(r, 3)]) * pow2(7 - ktab(r, 4) - kb);
      }
      __half2 s2 = __floats2half2_rn(lo, hi);
      const uint32_t su = *reinterpret_cast<uint32_t *>(&s2);
      rec[r] = pb ? su ^ 0x80008000u : su;  // hi lanes: q; lo lanes: -q
      rec[20 + r] = pb ? su : 0u;           // lo lanes: q; hi lanes: 0
    }
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      if (((ks + 2) & 3) != warp) continue;
      uint32_t a0 = 0u, a2 = 0u;
      if (g < G) {
        const uint32_t *qw = reinterpret_cast<const uint32_t *>(&qs[g][32 * tig + 4 * ks]);
        a0 = qw[0];
        a2 = qw[1];
      }
      rec[40 + 2 * ks] = a0;
      rec[41 + 2 * ks] = a2;
    }
  }
  return pick(tig);
}

// One 64-token block: K scores, online softmax and the P.V update of the running state
// (m_run, l_run, acc) for head tig of this lane.
template <bool REC>
__device__ __forceinline__ void block_step(const SStage &sg, const uint32_t *rec, float c1, int vword, uint32_t selL,
                                           uint32_t selH, int g, int tig, float &m_run, float &l_run,
                                           float (&acc)[8][4]) {
  constexpr float kLog2e = 1.4426950408889634f;
  constexpr float c2 = kScale;
  auto pow2 = [](int e) { return pow2f(e); };
  // ---- K weights of this block: W[r] = hi (even g) or lo (odd g) of q * scale * 2^(7-pos-kq)
  constexpr int KR = REC ? 16 : 18;  // K registers per token row of a lane group
  uint32_t W[KR];
  {
    uint32_t nat[16];
    const uint4 *ksv = reinterpret_cast<const uint4 *>(sg.ks + 32 * tig);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 v = ksv[i];
      nat[4 * i] = v.x;
      nat[4 * i + 1] = v.y;
      nat[4 * i + 2] = v.z;
      nat[4 * i + 3] = v.w;
    }
    uint32_t qa[20], qz[20];
    const uint4 *rq = reinterpret_cast<const uint4 *>(rec);
#pragma unroll
    for (int i = 0; i < (KR + 3) / 4; ++i) {
      const uint4 x = rq[i], y = rq[5 + i];
      qa[4 * i] = x.x, qa[4 * i + 1] = x.y, qa[4 * i + 2] = x.z, qa[4 * i + 3] = x.w;
      qz[4 * i] = y.x, qz[4 * i + 1] = y.y, qz[4 * i + 2] = y.z, qz[4 * i + 3] = y.w;
    }
#pragma unroll
    for (int r = 0; r < KR; ++r) {
      uint32_t b2;
      if constexpr (REC) {  // scales of channels 32 tig + r and 32 tig + 16 + r
        b2 = prmt(nat[r >> 1], nat[8 + (r >> 1)], (r & 1) ? 0x7632u : 0x5410u);
      } else {
        const uint32_t lo_src = ktab(r, 1) >= 0 ? nat[ktab(r, 1) >> 1] : 0u;
        const uint32_t hi_src = ktab(r, 3) >= 0 ? nat[ktab(r, 3) >> 1] : 0u;
        b2 = prmt(lo_src, hi_src, ksel(r));
      }
      W[r] = hfma2u(qz[r], b2, hmul2u(qa[r], b2));
    }
  }
  // ---- Delta_h = sum_c q_hc min_c on the tensor cores (rows = heads, every column alike)
  float dd[4] = {0.f, 0.f, 0.f, 0.f};
  {
    const uint4 *kmv = reinterpret_cast<const uint4 *>(sg.km + 32 * tig);
    const uint4 *rqd = reinterpret_cast<const uint4 *>(rec + 40);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 mv = kmv[i], qv = rqd[i];
      mma16816<__half>(dd, qv.x, 0u, qv.y, 0u, mv.x, mv.y);
      mma16816<__half>(dd, qv.z, 0u, qv.w, 0u, mv.z, mv.w);
    }
  }
  const float dlt = __shfl_sync(0xffffffffu, dd[0], 4 * tig) * c2;

  // ---- K: scores of tokens 16m+g and 16m+g+8 for head tig (two m-tiles at a time)
  float sc[4][4];
  {
    const uint32_t *kw = reinterpret_cast<const uint32_t *>(sg.kc);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t X0[2][6], X1[2][6];
#pragma unroll
      for (int mm = 0; mm < 2; ++mm) {
        const int m = 2 * half + mm;
        const uint32_t *p0 = kw + 12 * (16 * m + g) + 3 * tig, *p1 = p0 + 12 * 8;
        const uint32_t u0 = p0[0], u1 = p0[1], u2 = p0[2], v0 = p1[0], v1 = p1[1], v2 = p1[2];
        if constexpr (REC) {  // paired halves: windows of both 48-bit halves of the group at once
          X0[mm][0] = u0, X0[mm][1] = prmt(u0, u1, 0x6341u), X0[mm][2] = u1;
          X0[mm][3] = prmt(u1, u2, 0x6341u), X0[mm][4] = u2, X0[mm][5] = prmt(u2, u2, 0x3311u);
          X1[mm][0] = v0, X1[mm][1] = prmt(v0, v1, 0x6341u), X1[mm][2] = v1;
          X1[mm][3] = prmt(v1, v2, 0x6341u), X1[mm][4] = v2, X1[mm][5] = prmt(v2, v2, 0x3311u);
        } else {
          X0[mm][0] = u0, X0[mm][1] = __funnelshift_r(u0, u1, 8), X0[mm][2] = u1;
          X0[mm][3] = __funnelshift_r(u1, u2, 8), X0[mm][4] = u2, X0[mm][5] = u2 >> 8;
          X1[mm][0] = v0, X1[mm][1] = __funnelshift_r(v0, v1, 8), X1[mm][2] = v1;
          X1[mm][3] = __funnelshift_r(v1, v2, 8), X1[mm][4] = v2, X1[mm][5] = v2 >> 8;
        }
        sc[m][0] = sc[m][1] = sc[m][2] = sc[m][3] = 0.f;
      }
#pragma unroll
      for (int k = 0; k < KR / 2; ++k)
#pragma unroll
        for (int mm = 0; mm < 2; ++mm) {
          const int r0 = 2 * k, r1 = 2 * k + 1;
          if constexpr (REC) {
            constexpr uint32_t seven = 0x00070007u;
            const uint32_t m0 = seven << vpos(r0), m1 = seven << vpos(r1);
            mma16816<__half>(sc[2 * half + mm], X0[mm][vwin(r0)] & m0, X1[mm][vwin(r0)] & m0,
                             X0[mm][vwin(r1)] & m1, X1[mm][vwin(r1)] & m1, W[r0], W[r1]);
          } else {
            mma16816<__half>(sc[2 * half + mm], X0[mm][ktab(r0, 0)] & kmask(r0), X1[mm][ktab(r0, 0)] & kmask(r0),
                             X0[mm][ktab(r1, 0)] & kmask(r1), X1[mm][ktab(r1, 0)] & kmask(r1), W[r0], W[r1]);
          }
        }
    }
  }
  float s[4][2];
  float bm = -INFINITY;
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    s[m][0] = sg.ka[16 * m + g] * fmaf(sc[m][0] + sc[m][1], c1, dlt);
    s[m][1] = sg.ka[16 * m + g + 8] * fmaf(sc[m][2] + sc[m][3], c1, dlt);
    bm = fmaxf(bm, fmaxf(s[m][0], s[m][1]));
  }
  bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 4));
  bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 8));
  bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 16));
  const float m_new = fmaxf(m_run, bm);
  const float r = m_run == -INFINITY ? 0.f : ex2_neg((m_run - m_new) * kLog2e);
  const float mb = m_new * kLog2e;
  float psum = 0.f, wsum = 0.f;
  uint32_t PB[4][2];
#pragma unroll
  for (int m = 0; m < 4; ++m)
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float p = ex2_neg(fmaf(s[m][i], kLog2e, -mb));
      const float pv = p * sg.va[16 * m + g + 8 * i];
      psum += p;
      wsum += pv;
      PB[m][i] = movtrans(split_hilo(pv));
    }
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
  l_run = l_run * r + psum;  // this lane's tokens only: the head's sum is formed at the end
  m_run = m_new;
  if (!__all_sync(0xffffffffu, r == 1.f)) {
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i][0] *= r, acc[i][1] *= r, acc[i][2] *= r, acc[i][3] *= r;
  }

  // ---- V: D[mt] (channel slots 16g+2mt | 16g+2mt+1, head tig hi | lo) over the 64 tokens
  float D[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) D[i][0] = D[i][1] = D[i][2] = D[i][3] = 0.f;
  {
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      // P[pr][k]: window k of this lane's field for tokens 16ks + 2tig + 8pr (low half) and
      // the token after it (high half)
      uint32_t P[2][6];
      if constexpr (REC) {
        // paired rows: word 24 j + k = [token 2j half k | token 2j+1 half k], so both tokens'
        // windows come from the same three words (conflict-free: banks 24 tig + 3 g + c)
        const uint32_t *vw = reinterpret_cast<const uint32_t *>(sg.vc) + 3 * g;
#pragma unroll
        for (int pr = 0; pr < 2; ++pr) {
          const int j = 8 * ks + tig + 4 * pr;
          const uint32_t w0 = vw[24 * j], w1 = vw[24 * j + 1], w2 = vw[24 * j + 2];
          P[pr][0] = w0;
          P[pr][1] = prmt(w0, w1, 0x6341u);
          P[pr][2] = w1;
          P[pr][3] = prmt(w1, w2, 0x6341u);
          P[pr][4] = w2;
          P[pr][5] = prmt(w2, w2, 0x3311u);
        }
      } else {
        const uint32_t *vw = reinterpret_cast<const uint32_t *>(sg.vc) + vword;
        const int ta = 16 * ks + 2 * tig;
        uint32_t L[4], H[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int t = ta + (u & 1) + 8 * (u >> 1);  // ta, ta+1, ta+8, ta+9
          const uint32_t w0 = vw[12 * t], w1 = vw[12 * t + 1];
          L[u] = prmt(w0, w1, selL);
          H[u] = prmt(w0, w1, selH);
        }
#pragma unroll
        for (int pr = 0; pr < 2; ++pr) {
          const int x = 2 * pr, y = 2 * pr + 1;
          P[pr][0] = prmt(L[x], L[y], vsel(0));
          P[pr][1] = prmt(L[x], L[y], vsel(1));
          P[pr][2] = prmt(L[x], L[y], vsel(2));
          P[pr][3] = prmt(H[x], H[y], vsel(3));
          P[pr][4] = prmt(H[x], H[y], vsel(4));
          P[pr][5] = prmt(H[x], H[y], vsel(5));
        }
      }
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int i0 = 2 * mt, i1 = 2 * mt + 1;
        mma16816<__half>(D[mt], vop(P[0][vwin(i0)], i0), vop(P[0][vwin(i1)], i1), vop(P[1][vwin(i0)], i0),
                         vop(P[1][vwin(i1)], i1), PB[ks][0], PB[ks][1]);
      }
    }
  }
  // ---- epilogue: acc' += scale_c * D + min_c * 2^vunit(c) * sum_t p_t alpha_t
  {
    const uint4 *vsv = reinterpret_cast<const uint4 *>(sg.vs + 16 * g);
    const uint4 *vmv = reinterpret_cast<const uint4 *>(sg.vm + 16 * g);
    const uint4 s0 = vsv[0], s1 = vsv[1], n0 = vmv[0], n1 = vmv[1];
    const uint32_t sw[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const uint32_t nw[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const float2 bs = Elem<__half>::to_f2(sw[mt]), ms = Elem<__half>::to_f2(nw[mt]);
      acc[mt][0] = fmaf(bs.x, D[mt][0], fmaf(ms.x, wsum * pow2(vunit(2 * mt)), acc[mt][0]));
      acc[mt][1] = fmaf(bs.x, D[mt][1], acc[mt][1]);
      acc[mt][2] = fmaf(bs.y, D[mt][2], fmaf(ms.y, wsum * pow2(vunit(2 * mt + 1)), acc[mt][2]));
      acc[mt][3] = fmaf(bs.y, D[mt][3], acc[mt][3]);
    }
  }
}

// Combine the four warps' states of one chunk and write its partial (o, m, l) rows.
// row0 = b * hq + h * G (the chunk's first query head row); sync() synchronises the four
// warps (128 threads), tid is the thread's index among them.
template <typename Sync>
__device__ __forceinline__ void combine_chunk(SMerge &SM, int G, int tid, float m_run, float l_run,
                                              const float (&acc)[8][4], int64_t row0, int max_chunks, int chunk,
                                              float *part_o, float *part_ml, int &st, Sync sync) {
  constexpr float kLog2e = 1.4426950408889634f;
  const int lane = tid & 31, warp = tid >> 5, g = lane >> 2, tig = lane & 3;
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) l_run += __shfl_xor_sync(0xffffffffu, l_run, o);
  // a non-finite score or weight leaves the running sum non-finite (checked once per chunk;
  // the merge kernel also checks every output)
  if (tig < G && !isfinite(l_run)) st |= NSNKV_ST_OUTPUT_NONFINITE;
  MergeSmem &M = SM.part;
  sync();  // every warp is past its last block (the merge area may alias the block data)
  if (tig < G) {
    if (g == 0) {
      M.m[warp][tig] = m_run;
      M.l[warp][tig] = l_run;
    }
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int c = 16 * g + 2 * mt;
      M.acc[warp][tig][c] = (acc[mt][0] + acc[mt][1]) * pow2f(-vunit(2 * mt));
      M.acc[warp][tig][c + 1] = (acc[mt][2] + acc[mt][3]) * pow2f(-vunit(2 * mt + 1));
    }
  }
  sync();
  if (tid < G) {  // one thread per head: the warps' weights, the chunk's max and sum
    const int n = tid;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, M.m[w][n]);
    float l = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float wt = M.m[w][n] == -INFINITY ? 0.f : exp2f((M.m[w][n] - mx) * kLog2e);
      SM.wt[w][n] = wt;
      l += wt * M.l[w][n];
    }
    const int64_t row = (row0 + n) * max_chunks + chunk;
    part_ml[row * 2] = mx;
    part_ml[row * 2 + 1] = l;
  }
  sync();
  for (int e = tid; e < G * kDim; e += kThreads) {
    const int n = e / kDim, c = e % kDim;
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) o += SM.wt[w][n] * M.acc[w][n][c];
    const int64_t row = (row0 + n) * max_chunks + chunk;
    part_o[row * kDim + c] = o;
  }
}

}  // namespace s3

// REC: the codes are in the paged cache's block-record orders: K as paired halves (each
// 32-code group of a row stored as words [A half m | B half m]), V as paired rows (token
// rows 2j and 2j+1 interleaved at 16 bits).  Otherwise the reference's packed rows.
template <bool REC>
__global__ void __launch_bounds__(kThreads, 4) attn_sealed3_kernel(const AttnArgs a) {
  using namespace s3;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  SSmem &S = *reinterpret_cast<SSmem *>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, tig = lane & 3;
  pdl_wait();               // launched with a programmatic dependency on the kernel before it
  pdl_launch_dependents();  // the native-row chunks (next grid) may fill this grid's last wave
  const int chunk = blockIdx.x, h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int G = a.hq / a.h;
  const int nb = a.nblk ? a.nblk[b] : a.nblk_const;
  const int blk0 = chunk * a.chunk_blocks;
  if (blk0 >= nb) {
    if (chunk == 0) empty_unit<__half>(a, b, h);
    return;
  }
  const int nloc = min(nb - blk0, a.chunk_blocks);
  const __half *qb = static_cast<const __half *>(a.q) + (b * a.hq + static_cast<int64_t>(h) * G) * kDim;

  // Block li of the chunk goes to warp li % 4 and stage li % kRing; the warp that
  // finishes block li starts the copy of block li + kRing into the stage it frees, so a
  // stage is only ever refilled by its last reader.
  auto issue = [&](int li, int32_t page) {
    const int64_t bi = static_cast<int64_t>(h) * a.sh + static_cast<int64_t>(page) * a.sp;
    SStage &sg = S.u.stage[li % kRing];
    uint64_t *bar = &S.full[li % kRing][(li / kRing) & 1];
    S.nissued[li % kRing][(li / kRing) & 1] += 1;
    mbar_expect_tx(bar, sizeof(SStage));
    if (a.one_copy) {  // the block record: one copy (each cp.async.bulk issue can wait on the TMA queue)
      bulk_g2s(sg.kc, a.kc + bi * a.cs, sizeof(SStage), bar);
      return;
    }
    bulk_g2s(sg.kc, a.kc + bi * a.cs, kCB, bar);
    bulk_g2s(sg.vc, a.vc + bi * a.cs, kCB, bar);
    bulk_g2s(sg.km, blk_ptr(a.km, bi, a.ms), kDim * 2, bar);
    bulk_g2s(sg.ks, blk_ptr(a.ks, bi, a.ms), kDim * 2, bar);
    bulk_g2s(sg.vm, blk_ptr(a.vm, bi, a.ms), kDim * 2, bar);
    bulk_g2s(sg.vs, blk_ptr(a.vs, bi, a.ms), kDim * 2, bar);
    bulk_g2s(sg.ka, blk_ptr(a.ka, bi, a.ms), kBlock * 4, bar);
    bulk_g2s(sg.va, blk_ptr(a.va, bi, a.ms), kBlock * 4, bar);
  };
  // One round of global loads starts the CTA: q (8 bytes per thread) and the chunk's page
  // indices (warp 0, one coalesced load), staged in shared memory.  The copy issue never
  // waits on a global load: each cp.async.bulk is ordered after the loads before it, and
  // issuing one can itself stall on the TMA queue, so the first blocks are issued by every
  // warp (block li by warp li % 4) once the pages are in shared memory.
  uint2 qv = make_uint2(0u, 0u);
  if (tid < G * kDim / 4) qv = reinterpret_cast<const uint2 *>(qb)[tid];
  if (warp == 0) {
    int32_t pg = 0;
    if (lane < nloc) pg = a.table ? a.table[b * a.table_stride + blk0 + lane] : blk0 + lane;
    S.pages[lane] = pg;
    if (lane == 0) {
      S.failed = 0;
#pragma unroll
      for (int s = 0; s < kRing; ++s)
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          mbar_init(&S.full[s][x], 1);
          S.nissued[s][x] = 0;
        }
      fence_mbar_init();
    }
    __syncwarp();
  }
  if (tid < G * kDim / 4) reinterpret_cast<uint2 *>(&S.qs[0][0])[tid] = qv;
  __syncthreads();  // q and the pages staged; the ring initialised before any copy or wait
  if (lane == 0)
    for (int li = warp; li < kRing && li < nloc; li += kWarps) issue(li, S.pages[li]);
  __syncwarp();

  const int kq = build_records<REC>(S.qs, G, S.rec, lane, warp);
  __syncthreads();  // records written
  const float c1 = kScale * pow2f(17 + kq);
  const int vword = (3 * g - (g & 1)) >> 1;  // first word holding this lane's V field
  const uint32_t selL = (g & 1) ? 0x5432u : 0x3210u, selH = (g & 1) ? 0x7654u : 0x5432u;
  const uint32_t *rec = S.rec[lane];
  float m_run = -INFINITY, l_run = 0.f;
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  int st = 0;

  for (int li = warp; li < nloc; li += kWarps) {
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&S.full[li % kRing][(li / kRing) & 1], (li / (2 * kRing)) & 1,
                                                   a.status))) {
      if (lane == 0) S.failed = 1;
      break;
    }
    block_step<REC>(S.u.stage[li % kRing], rec, c1, vword, selL, selH, g, tig, m_run, l_run, acc);
    __syncwarp();
    if (lane == 0 && li + kRing < nloc) issue(li + kRing, S.pages[li + kRing]);
  }
  __syncthreads();
  if (S.failed) {  // a copy never landed: give every started copy a bounded chance to finish
    if (tid == 0)
      for (int s = 0; s < kRing; ++s)
        for (int x = 0; x < 2; ++x)
          if (S.nissued[s][x] > 0) mbar_wait_bounded(&S.full[s][x], (S.nissued[s][x] - 1) & 1, a.status);
  }
  combine_chunk(S.u.merge, G, tid, m_run, l_run, acc, b * a.hq + static_cast<int64_t>(h) * G, a.max_chunks, chunk,
                a.part_o, a.part_ml, st, [] { __syncthreads(); });
  if (st) set_status(a.status, st);
  unit_finish<__half>(a, b, h, smem_raw);
}



// ----------------------------------------------------------------- sealed INT3 blocks, K rounded like the bridge
// attn_sealed_kernel<T, NT>: the paged cache's default path (INT3 block records with
// per-token renorm factors, q / tails / output in T = fp16 or bf16, G <= 4 * NT query heads
// per kv head).  The reference bridge (restore_group(g, T), then SDPA) attends over
// restored rows rounded to T.  Rounding K moves a logit by up to ~2^-12 sum_c |q_c k_c| /
// sqrt(128), which with unscaled N(0,1) queries moves outputs by several 1e-3; rounding V
// moves an output by about 2^-12 of its own size.  So K is restored and rounded to T as
// the bridge rounds it, and V stays the exact fp32 restore:
//   K  per 16-token m-tile and register r (channels 32 tig + r and 32 tig + 16 + r of
//      tokens g and g + 8, both at position p = (3 r) mod 8 of their 16-bit windows): one
//      LOP3 turns the two codes into fp16 1024 + code * 2^p, one HSUB2 leaves code * 2^p
//      (exact), and one mma.m16n8k16 with A = [code * 2^p | 2^p] and a diagonal
//      B = [scale ; min] (both fp16, every product exact) gives 2^p * (min + scale * code)
//      in fp32.  Times alpha_t * 2^-p and rounded to T, that is the row restore_group stores
//      (its y = n * (d / ||d||) and this alpha_t * d differ in the order of two fp32
//      roundings, so a rounded value can differ by one unit of T in rare ties).  The
//      rounded pairs are the A fragments of the Q.K mma, B = q with each head in two
//      adjacent columns, so lane (g, tig) receives head tig's score in the layout the V
//      side of attn_sealed3_kernel consumes.
//   V  as in attn_sealed3_kernel: codes as fp16-subnormal operands against
//      B = p * alpha split into hi | lo, and an fp32 epilogue per block.
// NT = 2 serves G in 5..8: two head columns tiles, the K restore shared by both.
namespace s3 {

// d = A * B with fp32 accumulation from zero (m16n8k16, fp16 operands).
__device__ __forceinline__ void mma16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

template <typename T> __device__ __forceinline__ uint32_t round2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t round2<__half>(float lo, float hi) {
  __half2 p = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&p);
}
template <> __device__ __forceinline__ uint32_t round2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&p);
}

constexpr int kQf = 16;  // words of a lane's q fragments per head tile: 8 k-steps x (b0, b1)

// A block record of BITS-bit codes: K codes, min, scale, factors, then the same for V.
template <int BITS>
struct RStage {
  static constexpr int kCodeBytes = kBlock * kDim * BITS / 8;
  uint8_t kc[kCodeBytes];
  uint16_t km[kDim], ks[kDim];
  float ka[kBlock];
  uint8_t vc[kCodeBytes];
  uint16_t vm[kDim], vs[kDim];
  float va[kBlock];
};
static_assert(sizeof(RStage<3>) == sizeof(SStage) && sizeof(RStage<5>) == 11776, "record sizes");

// Code i (0..15) of a 16-code field starting at bit 0 of a 16-bit-window sequence: it sits
// at bit craw of byte window cwin.  For the fp16 operand forms the code must end at or
// below bit 10 of its window (code * 2^pos exact as 1024 + code * 2^pos, or as a
// subnormal); INT5 codes at window bits 6 and 7 are shifted down by 2 first (cshift),
// which moves the other half's low bits only into bits 14..15, outside the code's mask.
// For INT3 every shift is 0 and cpos == vpos, cwin == vwin.
template <int BITS> __host__ __device__ constexpr int cwin(int i) { return (BITS * i) >> 3; }
template <int BITS> __host__ __device__ constexpr int craw(int i) { return BITS * i - 8 * cwin<BITS>(i); }
template <int BITS> __host__ __device__ constexpr int cshift(int i) { return craw<BITS>(i) + BITS > 10 ? 2 : 0; }
template <int BITS> __host__ __device__ constexpr int cpos(int i) { return craw<BITS>(i) - cshift<BITS>(i); }
template <int BITS> __host__ __device__ constexpr uint32_t cmask(int i) {
  return ((1u << BITS) - 1u) * 0x00010001u << cpos<BITS>(i);
}
template <int BITS> __host__ __device__ constexpr int cunit(int i) {
  return cpos<BITS>(i) <= kVNormal ? cpos<BITS>(i) : cpos<BITS>(i) - 24;
}
static_assert(cwin<3>(13) == vwin(13) && cpos<3>(13) == vpos(13) && cunit<3>(5) == vunit(5), "INT3 forms");
// The code of register i in window word x (two tokens or two channels, one per half).
template <int BITS>
__device__ __forceinline__ uint32_t code2(uint32_t x, int i) {
  return (cshift<BITS>(i) ? x >> cshift<BITS>(i) : x) & cmask<BITS>(i);
}
// V operand of channel i (see vunit): normal fp16 code * 2^cpos up to kVNormal, else subnormal.
template <int BITS>
__device__ __forceinline__ uint32_t vopb(uint32_t x, int i) {
  const uint32_t c = code2<BITS>(x, i);
  return cpos<BITS>(i) <= kVNormal ? hsub2u(c | kMagic2, kMagic2) : c;
}
// The 2 BITS byte windows of a field held in BITS paired words w[0..BITS): window 2m is
// word m, window 2m+1 its high byte joined with the next word's low byte (per half).
template <int BITS>
__device__ __forceinline__ void windows(const uint32_t (&w)[BITS], uint32_t (&x)[2 * BITS]) {
#pragma unroll
  for (int m = 0; m < BITS; ++m) {
    x[2 * m] = w[m];
    x[2 * m + 1] = m + 1 < BITS ? prmt(w[m], w[m + 1], 0x6341u) : prmt(w[m], w[m], 0x3311u);
  }
}
template <int NT, int BITS> constexpr int kCtasPerSm = NT == 1 && BITS == 3 ? 3 : 2;

template <int NT, int BITS>
struct KSmem {
  union {
    RStage<BITS> stage[kRing];
    SMerge merge;  // after the last block of every warp
  } u;
  uint32_t qf[32][NT * kQf + 2];  // per lane: Q.K B fragments; stride 2 * odd words (conflict-free 64-bit loads)
  uint16_t qs[kHeads][kDim];      // this kv head's query rows (G <= 8), raw bits of T
  int32_t pages[kMaxChunk];
  uint64_t full[kRing][2];        // as in SSmem
  int32_t nissued[kRing][2];
  int32_t failed;
};

}  // namespace s3

template <typename T, int NT, int BITS>
__global__ void __launch_bounds__(kThreads, s3::kCtasPerSm<NT, BITS>) attn_sealed_kernel(const AttnArgs a) {
  using namespace s3;
  using Stg = RStage<BITS>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  KSmem<NT, BITS> &S = *reinterpret_cast<KSmem<NT, BITS> *>(smem_raw);
  constexpr float kLog2e = 1.4426950408889634f;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, tig = lane & 3;
  pdl_wait();               // launched with a programmatic dependency on the kernel before it
  pdl_launch_dependents();  // the native-row chunks (next grid) may fill this grid's last wave
  const int chunk = blockIdx.x, h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int G = a.hq / a.h;
  const int nb = a.nblk ? a.nblk[b] : a.nblk_const;
  const int blk0 = chunk * a.chunk_blocks;
  if (blk0 >= nb) {
    if (chunk == 0) empty_unit<T>(a, b, h);
    return;
  }
  const int nloc = min(nb - blk0, a.chunk_blocks);
  const uint16_t *qb = static_cast<const uint16_t *>(a.q) + (b * a.hq + static_cast<int64_t>(h) * G) * kDim;

  // Block li of the chunk goes to warp li % 4 and stage li % kRing (one copy of the block
  // record); the warp that finishes block li starts the copy of block li + kRing.
  auto issue = [&](int li, int32_t page) {
    const int64_t bi = static_cast<int64_t>(h) * a.sh + static_cast<int64_t>(page) * a.sp;
    Stg &sg = S.u.stage[li % kRing];
    uint64_t *bar = &S.full[li % kRing][(li / kRing) & 1];
    S.nissued[li % kRing][(li / kRing) & 1] += 1;
    mbar_expect_tx(bar, sizeof(Stg));
    bulk_g2s(sg.kc, a.kc + bi * a.cs, sizeof(Stg), bar);
  };
  // q (8 bytes per thread and pass) and the chunk's pages staged in shared memory
  uint2 qv[2] = {make_uint2(0u, 0u), make_uint2(0u, 0u)};
#pragma unroll
  for (int i = 0; i < 2; ++i)
    if (tid + i * kThreads < G * kDim / 4) qv[i] = reinterpret_cast<const uint2 *>(qb)[tid + i * kThreads];
  if (warp == 0) {
    int32_t pg = 0;
    if (lane < nloc) pg = a.table ? a.table[b * a.table_stride + blk0 + lane] : blk0 + lane;
    S.pages[lane] = pg;
    if (lane == 0) {
      S.failed = 0;
#pragma unroll
      for (int s = 0; s < kRing; ++s)
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          mbar_init(&S.full[s][x], 1);
          S.nissued[s][x] = 0;
        }
      fence_mbar_init();
    }
    __syncwarp();
  }
#pragma unroll
  for (int i = 0; i < 2; ++i)
    if (tid + i * kThreads < G * kDim / 4) reinterpret_cast<uint2 *>(&S.qs[0][0])[tid + i * kThreads] = qv[i];
  __syncthreads();  // q and the pages staged; the ring initialised before any copy or wait
  if (lane == 0)
    for (int li = warp; li < kRing && li < nloc; li += kWarps) issue(li, S.pages[li]);
  __syncwarp();

  // ---- Q.K B fragments of every lane (the same in every warp, each warp writing a quarter):
  // k-step p pairs registers r0 = BITS p mod 8 and r0 + 8 (both at window bit p; BITS is its
  // own inverse mod 8 for 3 and 5);
  // b0 = q[hd][32 tig + r0 | 32 tig + 16 + r0], b1 = the same for r0 + 8, column g -> head
  // hd = 4 nt + g / 2 (zero beyond G)
#pragma unroll
  for (int e = 0; e < NT * 8; ++e) {
    if ((e & 3) != warp) continue;
    const int nt = e >> 3, p = e & 7, r0 = (BITS * p) & 7;
    const int hd = 4 * nt + (g >> 1);
    uint32_t w0 = 0u, w1 = 0u;
    if (hd < G) {
      const uint16_t *qr = S.qs[hd] + 32 * tig;
      w0 = qr[r0] | (static_cast<uint32_t>(qr[16 + r0]) << 16);
      w1 = qr[r0 + 8] | (static_cast<uint32_t>(qr[24 + r0]) << 16);
    }
    S.qf[lane][nt * kQf + 2 * p] = w0;
    S.qf[lane][nt * kQf + 2 * p + 1] = w1;
  }
  __syncthreads();  // fragments written

  // diagonal entries of the restore MMA's B: lane (g, tig) with tig == g / 2 holds the scale
  // and min of channel dbase + r in half (g & 1); every other lane holds zeros
  const int dbase = 32 * (g >> 1) + 16 * (g & 1);
  const bool diag = tig == (g >> 1);
  const uint32_t selE = !diag ? 0x4444u : (g & 1) ? 0x1044u : 0x4410u;  // r even: low half of the pair word
  const uint32_t selO = !diag ? 0x4444u : (g & 1) ? 0x3244u : 0x4432u;  // r odd: high half
  const uint32_t *qfl = S.qf[lane];
  // This lane's Q.K B fragments: with one head tile kept in registers for the whole chunk;
  // with two read from shared memory at each use, which frees the 32 registers that
  // otherwise spill at 255 (cfg4 on one GPU: 82.4 against 86.1 us).
  uint32_t qreg[16];
  if constexpr (NT == 1) {
#pragma unroll
    for (int i = 0; i < 16; ++i) qreg[i] = qfl[i];
  }

  float m_run[NT], l_run[NT];
  // acc[nt][mt][i]: channel 16 g + 2 mt + i of head 4 nt + tig, in units of 2^vunit
  // (the hi and lo weight columns summed every block)
  float acc[NT][8][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m_run[nt] = -INFINITY;
    l_run[nt] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[nt][i][0] = acc[nt][i][1] = 0.f;
  }
  int st = 0;

  for (int li = warp; li < nloc; li += kWarps) {
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&S.full[li % kRing][(li / kRing) & 1], (li / (2 * kRing)) & 1,
                                                   a.status))) {
      if (lane == 0) S.failed = 1;
      break;
    }
    const Stg &sg = S.u.stage[li % kRing];

    // ---- K: restore, round to T, scores of tokens 16m+g and 16m+g+8 for head 4 nt + tig
    uint32_t bS[16], bM[16];  // register r's diagonal B fragments (scale, min) for this block
    {
      const uint4 s0 = *reinterpret_cast<const uint4 *>(sg.ks + dbase);
      const uint4 s1 = *reinterpret_cast<const uint4 *>(sg.ks + dbase + 8);
      const uint4 n0 = *reinterpret_cast<const uint4 *>(sg.km + dbase);
      const uint4 n1 = *reinterpret_cast<const uint4 *>(sg.km + dbase + 8);
      const uint32_t sw[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
      const uint32_t mw[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        bS[r] = prmt(sw[r >> 1], 0u, (r & 1) ? selO : selE);
        bM[r] = prmt(mw[r >> 1], 0u, (r & 1) ? selO : selE);
      }
    }
    float s[NT][4][2];
    {
      const uint32_t *kw = reinterpret_cast<const uint32_t *>(sg.kc);
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        // paired halves: token row t holds 4 BITS words, lane group tig's 32 channels in
        // words BITS tig .. BITS tig + BITS - 1 ([channels 0..15 half | channels 16..31 half])
        uint32_t X0[2 * BITS], X1[2 * BITS];
        {
          const uint32_t *p0 = kw + 4 * BITS * (16 * m + g) + BITS * tig, *p1 = p0 + 4 * BITS * 8;
          uint32_t u[BITS], v[BITS];
#pragma unroll
          for (int i = 0; i < BITS; ++i) u[i] = p0[i], v[i] = p1[i];
          windows<BITS>(u, X0);
          windows<BITS>(v, X1);
        }
        // alpha * 2^-q of tokens 16m+g (mgq) and 16m+g+8 (mhq), both halves alike, for the
        // k-step's operand bit q (0 at p = 0), carried along the k-steps as one value each
        float2 mgq = make_float2(sg.ka[16 * m + g], 0.f), mhq = make_float2(sg.ka[16 * m + g + 8], 0.f);
        mgq.y = mgq.x, mhq.y = mhq.x;
        float sc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const int r0 = (BITS * p) & 7;  // registers r0 and r0 + 8: window bit p, operand bit cpos(r0)
          const int q = cpos<BITS>(r0);
          const uint32_t pw = 0x3C003C00u + static_cast<uint32_t>(q) * 0x04000400u;  // fp16 2^q in both halves
          if (p > 0) {
            const float f = pow2f(cpos<BITS>((BITS * (p - 1)) & 7) - q);  // 0.5 except where INT5 shifts
            mgq = __fmul2_rn(mgq, make_float2(f, f));
            mhq = __fmul2_rn(mhq, make_float2(f, f));
          }
          uint32_t klo[2], khi[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int r = r0 + 8 * e;
            const uint32_t a0 = hsub2u(code2<BITS>(X0[cwin<BITS>(r)], r) | kMagic2, kMagic2);
            const uint32_t a1 = hsub2u(code2<BITS>(X1[cwin<BITS>(r)], r) | kMagic2, kMagic2);
            float d[4];
            mma16816_z(d, a0, a1, pw, pw, bS[r], bM[r]);
            const float2 y01 = __fmul2_rn(make_float2(d[0], d[1]), mgq);
            const float2 y23 = __fmul2_rn(make_float2(d[2], d[3]), mhq);
            klo[e] = round2<T>(y01.x, y01.y);
            khi[e] = round2<T>(y23.x, y23.y);
          }
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            uint32_t b0, b1;
            if constexpr (NT == 1) {
              b0 = qreg[2 * p], b1 = qreg[2 * p + 1];
            } else {  // a volatile load, so that the compiler does not hoist it back into registers
              asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];"
                           : "=r"(b0), "=r"(b1)
                           : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(qfl + nt * kQf + 2 * p))));
            }
            mma16816<T>(sc[nt], klo[0], khi[0], klo[1], khi[1], b0, b1);
          }
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          s[nt][m][0] = sc[nt][0] * kScale;
          s[nt][m][1] = sc[nt][2] * kScale;
        }
      }
    }

    // ---- per head tile: softmax, then V: D[mt] (channel slots 16g+2mt | 16g+2mt+1, head
    // 4 nt + tig hi | lo) over the 64 tokens with B = p * alpha_V split into fp16 hi | lo
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      uint32_t PB[4][2];
      float wsum = 0.f;
      {
        float bm = -INFINITY;
#pragma unroll
        for (int m = 0; m < 4; ++m) bm = fmaxf(bm, fmaxf(s[nt][m][0], s[nt][m][1]));
        bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 4));
        bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 8));
        bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 16));
        const float m_new = fmaxf(m_run[nt], bm);
        const float r = m_run[nt] == -INFINITY ? 0.f : ex2_neg((m_run[nt] - m_new) * kLog2e);
        const float mb = m_new * kLog2e;
        float psum = 0.f;
#pragma unroll
        for (int m = 0; m < 4; ++m)
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const float p = ex2_neg(fmaf(s[nt][m][i], kLog2e, -mb));
            const float pv = p * sg.va[16 * m + g + 8 * i];
            psum += p;
            wsum += pv;
            PB[m][i] = movtrans(split_hilo(pv));
          }
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
        l_run[nt] = l_run[nt] * r + psum;  // this lane's tokens only: the head's sum is formed at the end
        m_run[nt] = m_new;
        if (!__all_sync(0xffffffffu, r == 1.f)) {
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[nt][i][0] *= r, acc[nt][i][1] *= r;
        }
      }
      float D[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) D[i][0] = D[i][1] = D[i][2] = D[i][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        // paired rows: word 8 BITS j + k = [token 2j half k | token 2j+1 half k]; lane g's
        // 16 channels are halves BITS g .. BITS g + BITS - 1 of a row
        uint32_t P[2][2 * BITS];
        const uint32_t *vw = reinterpret_cast<const uint32_t *>(sg.vc) + BITS * g;
#pragma unroll
        for (int pr = 0; pr < 2; ++pr) {
          const int j = 8 * ks + tig + 4 * pr;
          uint32_t w[BITS];
#pragma unroll
          for (int i = 0; i < BITS; ++i) w[i] = vw[8 * BITS * j + i];
          windows<BITS>(w, P[pr]);
        }
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int i0 = 2 * mt, i1 = 2 * mt + 1;
          mma16816<__half>(D[mt], vopb<BITS>(P[0][cwin<BITS>(i0)], i0), vopb<BITS>(P[0][cwin<BITS>(i1)], i1),
                           vopb<BITS>(P[1][cwin<BITS>(i0)], i0), vopb<BITS>(P[1][cwin<BITS>(i1)], i1), PB[ks][0],
                           PB[ks][1]);
        }
      }
      // epilogue: acc' += scale_c * D + min_c * 2^vunit(c) * sum_t p_t alpha_t
      const uint4 *vsv = reinterpret_cast<const uint4 *>(sg.vs + 16 * g);
      const uint4 *vmv = reinterpret_cast<const uint4 *>(sg.vm + 16 * g);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const uint4 sv = vsv[half], mv = vmv[half];
        const uint32_t sw4[4] = {sv.x, sv.y, sv.z, sv.w}, mw4[4] = {mv.x, mv.y, mv.z, mv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int mt = 4 * half + q;
          const float2 bs = Elem<__half>::to_f2(sw4[q]), ms = Elem<__half>::to_f2(mw4[q]);
          const float w0 = wsum * __int_as_float((127 + cunit<BITS>(2 * mt)) << 23);
          const float w1 = wsum * __int_as_float((127 + cunit<BITS>(2 * mt + 1)) << 23);
          acc[nt][mt][0] = fmaf(bs.x, D[mt][0] + D[mt][1], fmaf(ms.x, w0, acc[nt][mt][0]));
          acc[nt][mt][1] = fmaf(bs.y, D[mt][2] + D[mt][3], fmaf(ms.y, w1, acc[nt][mt][1]));
        }
      }
    }
    __syncwarp();
    if (lane == 0 && li + kRing < nloc) issue(li + kRing, S.pages[li + kRing]);
  }
  __syncthreads();
  if (S.failed) {  // a copy never landed: give every started copy a bounded chance to finish
    if (tid == 0)
      for (int s2 = 0; s2 < kRing; ++s2)
        for (int x = 0; x < 2; ++x)
          if (S.nissued[s2][x] > 0) mbar_wait_bounded(&S.full[s2][x], (S.nissued[s2][x] - 1) & 1, a.status);
    __syncthreads();  // the stages are reused below
  }

  // ---- combine the four warps and write this chunk's partial
  MergeSmem &M = S.u.merge.part;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float l = l_run[nt];
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    const int hd = 4 * nt + tig;
    // a non-finite score or weight leaves the running sum non-finite (checked once per chunk;
    // the merge kernel also checks every output)
    if (hd < G && !isfinite(l)) st |= NSNKV_ST_OUTPUT_NONFINITE;
    if (hd < G) {
      if (g == 0) {
        M.m[warp][hd] = m_run[nt];
        M.l[warp][hd] = l;
      }
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int c = 16 * g + 2 * mt;
        M.acc[warp][hd][c] = acc[nt][mt][0] * __int_as_float((127 - cunit<BITS>(2 * mt)) << 23);
        M.acc[warp][hd][c + 1] = acc[nt][mt][1] * __int_as_float((127 - cunit<BITS>(2 * mt + 1)) << 23);
      }
    }
  }
  __syncthreads();
  if (tid < G) {  // one thread per head: the warps' weights, the chunk's max and sum
    const int n = tid;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, M.m[w][n]);
    float l = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float wt = M.m[w][n] == -INFINITY ? 0.f : exp2f((M.m[w][n] - mx) * kLog2e);
      S.u.merge.wt[w][n] = wt;
      l += wt * M.l[w][n];
    }
    const int64_t row = (b * a.hq + static_cast<int64_t>(h) * G + n) * a.max_chunks + chunk;
    a.part_ml[row * 2] = mx;
    a.part_ml[row * 2 + 1] = l;
  }
  __syncthreads();
  for (int e = tid; e < G * kDim; e += kThreads) {
    const int n = e / kDim, c = e % kDim;
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) o += S.u.merge.wt[w][n] * M.acc[w][n][c];
    const int64_t row = (b * a.hq + static_cast<int64_t>(h) * G + n) * a.max_chunks + chunk;
    a.part_o[row * kDim + c] = o;
  }
  if (st) set_status(a.status, st);
  unit_finish<T>(a, b, h, smem_raw);
}

// ----------------------------------------------------------------- host side
static int chunk_blocks_for(int64_t batch, int h, int32_t max_blocks, int32_t max_tail) {
  // Aim for >= 4 CTAs per SM (148 SMs) while keeping the partials small.
  const int64_t units = batch * h;
  const int64_t target = 148 * 12;
  const int64_t work = max_blocks + (static_cast<int64_t>(max_tail) + 1 + kBlock - 1) / kBlock;
  int64_t per_unit = (target + units - 1) / units;  // desired chunks per (seq, head)
  int64_t ch = (work + per_unit - 1) / per_unit;
  ch = (ch + 3) / 4 * 4;  // whole rounds of the sealed kernel's four warps
  if (ch < 4) ch = 4;
  if (ch > 16) ch = 16;
  return static_cast<int>(ch);
}

// The sealed INT3 kernels' chunks: about one CTA per resident slot (148 SMs x per_sm) for
// the average sequence, in multiples of 4 blocks (one round of its four warps), up to 32
// blocks and never below the restore kernel's chunks (the workspace is sized for those).
// blocks_total, the sum of n_blocks when the caller knows it, gives the average; without
// it the bound max_blocks stands in, which undersizes the grid when lengths differ.
static int s3_chunk_blocks(int64_t batch, int h, int32_t max_blocks, int32_t max_tail, int per_sm,
                           int64_t blocks_total) {
  const int64_t units = batch * h;
  const int64_t target = 148 * per_sm;
  const int64_t avg = blocks_total > 0 ? (blocks_total + batch - 1) / batch : max_blocks;
  const int64_t work = avg + (static_cast<int64_t>(max_tail) + 1 + kBlock - 1) / kBlock;
  const int64_t per_unit = (target + units - 1) / units;
  int64_t ch = (work + per_unit - 1) / per_unit;
  ch = (ch + 3) / 4 * 4;
  if (ch < 4) ch = 4;
  if (ch > 32) ch = 32;
  const int64_t floor_ch = chunk_blocks_for(batch, h, max_blocks, max_tail);
  ch = std::max<int64_t>(ch, floor_ch);
  if (batch > 1) {
    // Under two waves the rounding of each sequence's last chunk decides: a sequence ends
    // half a chunk past its blocks on average, so a grid sized for the average sequence can
    // land just past a wave, whose last CTAs then run alone (8 cfg2 sequences, one rank of
    // 8: 624-640 CTAs of 16 blocks for 592 slots).  Here the multiple of 4 from min(ch, 16)
    // to 32 that minimises waves x (c + 2 blocks of start-up) wins, with the expected CTA
    // count units x (avg / c + 1/2).  On B200: a rank of 8, 20 blocks 31.5-32.0 us against
    // 37.0-38.8 at 16; a rank of 4, 20 blocks 51.7 us against 59.1 at 32.  From two waves
    // up, later CTAs fill the slots as earlier ones end, and the chunk above stays.
    const auto ctas = [&](int64_t c) { return (units * (2 * avg + c) + 2 * c - 1) / (2 * c); };
    if (ctas(ch) < 2 * target) {
      int64_t best = ch, best_cost = (ctas(ch) + target - 1) / target * (ch + 2);
      for (int64_t c = std::max<int64_t>(std::min<int64_t>(ch, 16), (floor_ch + 3) / 4 * 4); c <= 32; c += 4) {
        const int64_t cost = (ctas(c) + target - 1) / target * (c + 2);
        if (cost < best_cost) best = c, best_cost = cost;
      }
      ch = best;
    }
  }
  if (batch == 1) {
    // One sequence: every CTA but the last of each head runs c blocks.  Candidates start at
    // about two CTAs per SM, at most 16 blocks (fewer, longer chunks cost fewer CTA starts
    // and a shorter merge; on B200, cfg1 ran fastest at 12-16 blocks); the multiple of 4
    // that minimises waves x (c + 2 blocks of start-up) wins (cfg4 on one GPU: 28 blocks
    // fill two waves exactly where 32 leave the second 73% full).
    const int64_t c0 = (units * max_blocks + 2 * 148 - 1) / (2 * 148);
    const int64_t lo = std::max<int64_t>(std::min<int64_t>((c0 + 3) / 4 * 4, 16), (floor_ch + 3) / 4 * 4);
    int64_t best = lo, best_cost = INT64_MAX;
    for (int64_t c = lo; c <= 32; c += 4) {
      const int64_t ctas = units * ((max_blocks + c - 1) / c);
      const int64_t cost = (ctas + target - 1) / target * (c + 2);
      if (cost < best_cost) best = c, best_cost = cost;
    }
    ch = best;
  }
  return static_cast<int>(ch);
}

// attn_sealed_kernel for BITS, the dtype and the head-tile count, with its shared memory
// and resident CTAs per SM.
template <int BITS>
static void sealed_round_kernel(int dtype, bool wide, void (*&kern)(const AttnArgs), size_t &smem, int &per_sm) {
  per_sm = wide ? s3::kCtasPerSm<2, BITS> : s3::kCtasPerSm<1, BITS>;
  smem = wide ? sizeof(s3::KSmem<2, BITS>) : sizeof(s3::KSmem<1, BITS>);
  if (dtype == NSNKV_F16)
    kern = wide ? attn_sealed_kernel<__half, 2, BITS> : attn_sealed_kernel<__half, 1, BITS>;
  else
    kern = wide ? attn_sealed_kernel<__nv_bfloat16, 2, BITS> : attn_sealed_kernel<__nv_bfloat16, 1, BITS>;
}

// The workspace starts with the fused merge's arrival words (one per unit), then the partials.
static int64_t arrive_bytes(int64_t batch, int h) { return (batch * h * 8 + 255) / 256 * 256; }

static std::atomic<uint32_t> g_attn_epoch{0};  // arrival epochs: one per decode call
static thread_local int g_attn_launches = 0;   // kernels the calling thread's last decode call launched

int attn_last_launches() { return g_attn_launches; }

// Merge in the chunk kernels (unit_finish) or in attn_merge_kernel.  The fused merge
// saves the merge launch and its wait, which matters when the chunk grid is about one wave
// (small batches); over several waves the separate merge is cheaper than the per-CTA
// arrival and the serial last-CTA merge (measured on B200 over the batched decode
// benchmark's sequences: decode steps 7% faster at 8 sequences, 2.6% slower at 64).
static bool fuse_merge(int64_t batch, int h, int32_t max_blocks, int32_t max_tail, int32_t ch, int32_t max_chunks,
                       int per_sm, int64_t blocks_total) {
  // few units (one sequence's kv heads) leave each last CTA a long serial merge, where the
  // merge kernel spreads the query heads over CTAs (cfg1: 31.7 against 25.6 us)
  if (max_chunks > kFusedChunks || batch * h < 32) return false;
  const int64_t avg = blocks_total > 0 ? (blocks_total + batch - 1) / batch : max_blocks;
  const int64_t tail_chunks = (static_cast<int64_t>(max_tail) + 1 + static_cast<int64_t>(ch) * kBlock - 1) /
                              (static_cast<int64_t>(ch) * kBlock);
  const int64_t ctas = batch * h * ((avg + ch - 1) / ch + tail_chunks);
  return ctas <= 2 * 148 * static_cast<int64_t>(per_sm);
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
  return arrive_bytes(batch, h) + batch * hq * mc * (kDim + 2) * static_cast<int64_t>(sizeof(float));
}

}  // extern "C"

namespace nsnkv {
static int decode_attn_impl(int64_t batch, int hq, int h, int bits, int dtype, const void *q, const uint8_t *k_codes,
                            const uint16_t *k_norm, const uint16_t *k_min, const uint16_t *k_scale,
                            const uint8_t *v_codes, const uint16_t *v_norm, const uint16_t *v_min,
                            const uint16_t *v_scale, const float *k_alpha, const float *v_alpha, int64_t blk_bytes,
                            int flags, int64_t blk_stride_head, int64_t blk_stride_page, const int32_t *block_table,
                            int64_t table_stride, const int32_t *n_blocks, int32_t n_blocks_const, int32_t max_blocks,
                            int64_t blocks_total, void *k_tail, void *v_tail, int64_t tail_stride_seq,
                            int64_t tail_stride_head,
                            const int32_t *tail_len, int32_t tail_len_const, int32_t max_tail, const void *k_new,
                            const void *v_new, void *out, float *out_f32, float *lse, void *workspace,
                            int64_t workspace_bytes, int32_t *status, void *stream) {
  if (batch <= 0 || hq <= 0 || h <= 0 || hq % h != 0 || max_blocks < 0 || max_tail < 0) return NSNKV_ERR_ARG;
  if (bits < 3 || bits > 5 || (dtype != NSNKV_F16 && dtype != NSNKV_BF16)) return NSNKV_ERR_ARG;
  if (!q || !out || !status || !workspace || !aligned16(q) || !aligned16(out) || !aligned16(workspace))
    return NSNKV_ERR_ARG;
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
  const int64_t cb = code_bytes(bits);
  if (blk_bytes != 0 && (blk_bytes < cb || blk_bytes % 16 != 0)) return NSNKV_ERR_ARG;
  if (flags & ~(NSNKV_ATTN_RECORD_ORDER | NSNKV_ATTN_EXACT)) return NSNKV_ERR_ARG;
  const bool rec_order = (flags & NSNKV_ATTN_RECORD_ORDER) != 0, exact = (flags & NSNKV_ATTN_EXACT) != 0;

  AttnArgs a{};
  a.cs = blk_bytes ? blk_bytes : cb;
  a.ms = blk_bytes ? blk_bytes : kDim * 2;
  {  // K record then V record, contiguous: [codes | min | scale | factors] twice
    const uint8_t *r = k_codes;
    const auto at = [&](const void *p, int64_t off) { return static_cast<const void *>(r + off) == p; };
    a.one_copy = blk_bytes == 2 * (cb + 768) && at(k_min, cb) && at(k_scale, cb + 256) && at(k_alpha, cb + 512) &&
                 at(v_codes, cb + 768) && at(v_min, 2 * cb + 768) && at(v_scale, 2 * cb + 1024) &&
                 at(v_alpha, 2 * cb + 1280);
  }
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
  a.arrive = static_cast<unsigned long long *>(workspace);
  float *ws = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + arrive_bytes(batch, h));
  a.part_o = ws;
  a.part_ml = ws + batch * hq * static_cast<int64_t>(a.max_chunks) * kDim;
  a.status = status;
  a.epoch = g_attn_epoch.fetch_add(1u, std::memory_order_relaxed);
  a.out = out;
  a.out_f32 = out_f32;
  a.lse = lse;
  const int G = hq / h;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = NSNKV_OK;
  // Sealed blocks with renorm factors go to a tensor-core kernel: exact restore
  // (attn_sealed3_kernel: INT3, fp16, G <= 4, either code order) or, by default, K rounded
  // to the cache dtype as the bridge rounds it (attn_sealed_kernel: INT3 or INT5 in the
  // record orders, G <= 8).
  const bool sealed_exact = k_alpha && v_alpha && exact && bits == 3 && dtype == NSNKV_F16 && G <= 4;
  const bool sealed_round = k_alpha && v_alpha && !exact && rec_order && (bits == 3 || bits == 5) && G <= kHeads;
  const bool sealed_path = sealed_exact || sealed_round;
  if (rec_order && max_blocks > 0 && !sealed_path) return NSNKV_ERR_UNSUPPORTED;  // record orders: tensor-core kernels only
  if (exact && max_blocks > 0 && !sealed_exact) return NSNKV_ERR_UNSUPPORTED;
  if (sealed_path && max_blocks > 0) {
    // sealed chunks on a tensor-core kernel, native-row chunks on attn_native_rows_kernel
    if (!aligned16(k_alpha) || !aligned16(v_alpha)) return NSNKV_ERR_ARG;
    if (sealed_round && !a.one_copy) return NSNKV_ERR_ARG;  // the rounding kernel moves whole block records
    a.ka = k_alpha;
    a.va = v_alpha;
    size_t smem = sizeof(s3::SSmem);
    void (*kern)(const AttnArgs) = rec_order ? attn_sealed3_kernel<true> : attn_sealed3_kernel<false>;
    int per_sm = 4;
    if (sealed_round) {
      const bool wide = G > 4;
      if (bits == 3)
        sealed_round_kernel<3>(dtype, wide, kern, smem, per_sm);
      else
        sealed_round_kernel<5>(dtype, wide, kern, smem, per_sm);
    }
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return NSNKV_ERR_CUDA;
    // whole chunks of up to 32 blocks (8 per warp) amortise the per-CTA set-up; fewer chunks
    // than nsnkv_decode_attn_workspace_bytes() sized for, so the same workspace holds them
    a.chunk_blocks = s3_chunk_blocks(batch, h, max_blocks, max_tail, per_sm, n_blocks ? blocks_total : 0);
    a.max_chunks = max_chunks_for(max_blocks, max_tail, a.chunk_blocks);
    a.part_ml = a.part_o + batch * hq * static_cast<int64_t>(a.max_chunks) * kDim;
    a.fused = fuse_merge(batch, h, max_blocks, max_tail, a.chunk_blocks, a.max_chunks, per_sm,
                         n_blocks ? blocks_total : 0);
    // sealed chunks here, native-row chunks on attn_partial_kernel, then the merge kernel
    const int sealed_chunks = (max_blocks + a.chunk_blocks - 1) / a.chunk_blocks;
    {  // programmatic dependency on the kernel before it (it waits on entry)
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3(sealed_chunks, h, static_cast<unsigned>(batch));
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = st;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaLaunchKernelEx(&cfg, kern, a) != cudaSuccess) return NSNKV_ERR_LAUNCH;
    }
    if (cudaGetLastError() != cudaSuccess) return NSNKV_ERR_LAUNCH;
    if (any_tail) {  // native-row chunks, overlapping the sealed grid's last wave
      a.raw_only = 1;
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3(a.max_chunks - sealed_chunks, h, static_cast<unsigned>(batch));
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = sizeof(RawSmem);
      cfg.stream = st;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      const auto tails = dtype == NSNKV_F16 ? attn_native_rows_kernel<__half> : attn_native_rows_kernel<__nv_bfloat16>;
      if (cudaLaunchKernelEx(&cfg, tails, a) != cudaSuccess) return NSNKV_ERR_LAUNCH;
      rc = cudaGetLastError() == cudaSuccess ? NSNKV_OK : NSNKV_ERR_LAUNCH;
    }
  } else {
    a.fused = fuse_merge(batch, h, max_blocks, max_tail, a.chunk_blocks, a.max_chunks, 3, 0);
    dim3 grid(a.max_chunks, h, static_cast<unsigned>(batch));
    rc = dtype == NSNKV_F16 ? dispatch_bits<__half>(bits, G, a, grid, st)
                            : dispatch_bits<__nv_bfloat16>(bits, G, a, grid, st);
  }
  if (rc != NSNKV_OK) return rc;
  // kernels launched by this call: the chunk grid(s), then the merge unless fused
  g_attn_launches = 1 + (sealed_path && max_blocks > 0 && any_tail ? 1 : 0) + (a.fused ? 0 : 1);
  if (a.fused) return NSNKV_OK;  // the last chunk CTA of every unit merged it
  // the merge launches with a programmatic dependency on the kernel before it and waits
  // for it on entry, so its launch overlaps that kernel's end
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(hq, static_cast<unsigned>(batch));
  cfg.blockDim = dim3(kDim);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (dtype == NSNKV_F16)
    e = cudaLaunchKernelEx(&cfg, attn_merge_kernel<__half>, a, G, static_cast<__half *>(out), out_f32, lse);
  else
    e = cudaLaunchKernelEx(&cfg, attn_merge_kernel<__nv_bfloat16>, a, G, static_cast<__nv_bfloat16 *>(out), out_f32,
                           lse);
  return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? NSNKV_OK : NSNKV_ERR_LAUNCH;
}
}  // namespace nsnkv

extern "C" {

int nsnkv_decode_attn(int64_t batch, int hq, int h, int bits, int dtype, const void *q, const uint8_t *k_codes,
                      const uint16_t *k_norm, const uint16_t *k_min, const uint16_t *k_scale, const uint8_t *v_codes,
                      const uint16_t *v_norm, const uint16_t *v_min, const uint16_t *v_scale, int64_t blk_stride_head,
                      int64_t blk_stride_page, const int32_t *block_table, int64_t table_stride,
                      const int32_t *n_blocks, int32_t n_blocks_const, int32_t max_blocks, void *k_tail, void *v_tail,
                      int64_t tail_stride_seq, int64_t tail_stride_head, const int32_t *tail_len,
                      int32_t tail_len_const, int32_t max_tail, const void *k_new, const void *v_new, void *out,
                      float *out_f32, float *lse, void *workspace, int64_t workspace_bytes, int32_t *status,
                      void *stream) {
  return decode_attn_impl(batch, hq, h, bits, dtype, q, k_codes, k_norm, k_min, k_scale, v_codes, v_norm, v_min,
                          v_scale, nullptr, nullptr, 0, 0, blk_stride_head, blk_stride_page, block_table, table_stride,
                          n_blocks, n_blocks_const, max_blocks, 0, k_tail, v_tail, tail_stride_seq, tail_stride_head,
                          tail_len, tail_len_const, max_tail, k_new, v_new, out, out_f32, lse, workspace,
                          workspace_bytes, status, stream);
}

int nsnkv_decode_attn_alpha(int64_t batch, int hq, int h, int bits, int dtype, const void *q,
                            const uint8_t *k_codes, const uint16_t *k_norm, const uint16_t *k_min,
                            const uint16_t *k_scale, const uint8_t *v_codes, const uint16_t *v_norm,
                            const uint16_t *v_min, const uint16_t *v_scale, const float *k_alpha,
                            const float *v_alpha, int64_t blk_bytes, int flags, int64_t blk_stride_head,
                            int64_t blk_stride_page, const int32_t *block_table, int64_t table_stride,
                            const int32_t *n_blocks, int32_t n_blocks_const, int32_t max_blocks,
                            int64_t blocks_total, void *k_tail, void *v_tail, int64_t tail_stride_seq,
                            int64_t tail_stride_head, const int32_t *tail_len, int32_t tail_len_const,
                            int32_t max_tail, const void *k_new, const void *v_new, void *out, float *out_f32,
                            float *lse, void *workspace, int64_t workspace_bytes, int32_t *status, void *stream) {
  if ((k_alpha == nullptr) != (v_alpha == nullptr) || blocks_total < 0) return NSNKV_ERR_ARG;
  return decode_attn_impl(batch, hq, h, bits, dtype, q, k_codes, k_norm, k_min, k_scale, v_codes, v_norm, v_min,
                          v_scale, k_alpha, v_alpha, blk_bytes, flags, blk_stride_head, blk_stride_page,
                          block_table, table_stride, n_blocks, n_blocks_const, max_blocks, blocks_total, k_tail,
                          v_tail, tail_stride_seq, tail_stride_head, tail_len, tail_len_const, max_tail, k_new, v_new,
                          out, out_f32, lse, workspace, workspace_bytes, status, stream);
}

static int merge_shards_launch(int n_shards, int64_t rows, const float *o, int64_t o_stride, const float *lse,
                               int64_t lse_stride, int dtype, void *out, float *out_f32, float *lse_out,
                               int32_t *status, void *stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(rows);
  if (dtype == NSNKV_F16)
    merge_shards_kernel<__half><<<grid, kDim, 0, st>>>(n_shards, rows, o, o_stride, lse, lse_stride,
                                                       static_cast<__half *>(out), out_f32, lse_out, status);
  else if (dtype == NSNKV_BF16)
    merge_shards_kernel<__nv_bfloat16><<<grid, kDim, 0, st>>>(n_shards, rows, o, o_stride, lse, lse_stride,
                                                              static_cast<__nv_bfloat16 *>(out), out_f32, lse_out,
                                                              status);
  else
    return NSNKV_ERR_ARG;
  return cudaGetLastError() == cudaSuccess ? NSNKV_OK : NSNKV_ERR_LAUNCH;
}

int nsnkv_merge_shards(int n_shards, int64_t rows, const float *o, const float *lse, int dtype, void *out,
                       float *out_f32, float *lse_out, int32_t *status, void *stream) {
  if (n_shards <= 0 || rows <= 0 || rows > 0x7FFFFFFF || !o || !lse || !out || !status) return NSNKV_ERR_ARG;
  return merge_shards_launch(n_shards, rows, o, rows * kDim, lse, rows, dtype, out, out_f32, lse_out, status, stream);
}

int nsnkv_merge_shard_records(int n_shards, int64_t rows, const float *records, int64_t record_stride, int dtype,
                              void *out, float *out_f32, float *lse_out, int32_t *status, void *stream) {
  if (n_shards <= 0 || rows <= 0 || rows > 0x7FFFFFFF || !records || !out || !status) return NSNKV_ERR_ARG;
  if (record_stride < rows * (kDim + 1)) return NSNKV_ERR_ARG;
  return merge_shards_launch(n_shards, rows, records, record_stride, records + rows * kDim, record_stride, dtype, out,
                             out_f32, lse_out, status, stream);
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
