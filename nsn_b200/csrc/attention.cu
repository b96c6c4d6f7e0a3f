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

template <int BITS, typename T>
__global__ void __launch_bounds__(kThreads, 3) attn_partial_kernel(const AttnArgs a) {
  constexpr int CB = code_bytes(BITS);
  extern __shared__ __align__(128) uint8_t smem_raw[];
  AttnSmem<BITS> &S = *reinterpret_cast<AttnSmem<BITS> *>(smem_raw);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tig = lane & 3, cbase = 32 * tig, mi = meta_index(cbase);
  const int t0 = 16 * warp + g, t1 = t0 + 8;
  const int chunk = blockIdx.x, h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int G = a.hq / a.h;

  const int nb = a.nblk ? a.nblk[b] : a.nblk_const;
  const int tl = a.tlen ? a.tlen[b] : a.tlen_const;
  const int tail_total = tl + (a.knew ? 1 : 0);
  const int n_sealed_chunks = (nb + a.chunk_blocks - 1) / a.chunk_blocks;
  const int raw_per_chunk = a.chunk_blocks * kBlock;
  const int n_chunks = n_sealed_chunks + (tail_total + raw_per_chunk - 1) / raw_per_chunk;
  if (chunk >= n_chunks) return;
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

  if (!is_raw) {
    const int blk0 = chunk * a.chunk_blocks;
    const int nloc = min(nb, blk0 + a.chunk_blocks) - blk0;
    auto issue = [&](int i, int s) {
      const int32_t page = a.table ? a.table[b * a.table_stride + i] : i;
      const int64_t bi = static_cast<int64_t>(h) * a.sh + static_cast<int64_t>(page) * a.sp;
      Stage<BITS> &sg = S.stage[s];
      mbar_expect_tx(&S.full[s], 2 * CB + 2 * (kBlock * 2 + 2 * kDim * 2));
      bulk_g2s(sg.kc, a.kc + bi * CB, CB, &S.full[s]);
      bulk_g2s(sg.vc, a.vc + bi * CB, CB, &S.full[s]);
      bulk_g2s(sg.kn, a.kn + bi * kBlock, kBlock * 2, &S.full[s]);
      bulk_g2s(sg.km, a.km + bi * kDim, kDim * 2, &S.full[s]);
      bulk_g2s(sg.ks, a.ks + bi * kDim, kDim * 2, &S.full[s]);
      bulk_g2s(sg.vn, a.vn + bi * kBlock, kBlock * 2, &S.full[s]);
      bulk_g2s(sg.vm, a.vm + bi * kDim, kDim * 2, &S.full[s]);
      bulk_g2s(sg.vs, a.vs + bi * kDim, kDim * 2, &S.full[s]);
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

// ----------------------------------------------------------------- host side
static int chunk_blocks_for(int64_t batch, int h, int32_t max_blocks, int32_t max_tail) {
  // Aim for >= 4 CTAs per SM (148 SMs) while keeping the partials small.
  const int64_t units = batch * h;
  const int64_t target = 148 * 12;
  const int64_t work = max_blocks + (static_cast<int64_t>(max_tail) + 1 + kBlock - 1) / kBlock;
  int64_t per_unit = (target + units - 1) / units;  // desired chunks per (seq, head)
  int64_t ch = (work + per_unit - 1) / per_unit;
  if (ch < 4) ch = 4;
  if (ch > 16) ch = 16;
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
