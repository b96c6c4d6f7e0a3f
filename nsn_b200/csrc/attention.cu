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

constexpr int kThreads = 128;    // 4 warps: 4 x 16 tokens of a 64-token block
constexpr int kHeads = 8;        // MMA N: query heads per kv head (G <= 8)
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

// Per-block fp32 metadata in the form the restore uses: with x = 1 + code * 2^-BITS
// (the code dropped into the top mantissa bits of 1.0f),
//   d = min + scale*code = b*x + a,  b = scale * 2^BITS,  a = min - b.
struct MetaF {
  float ka[kMetaRow], kb[kMetaRow], va[kMetaRow], vb[kMetaRow];
};

template <int BITS>
struct AttnSmem {
  Stage<BITS> stage[kStages];
  MetaF meta[2];
  uint16_t v16[kBlock][kVRow];  // restored V tile in the bridge dtype
  float sc[kHeads][kBlock];     // scores of the current tile
  uint64_t full[kStages];
};

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ int meta_index(int c) { return c + (c >> 5) * 4; }

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
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void *smem_row) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem_row));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

__device__ __forceinline__ bool finite2(float2 v) { return isfinite(v.x) && isfinite(v.y); }

// Load the packed bits of this lane's 32 channels of token t, aligned so that
// channel j's code starts at bit BITS*j of the returned word array.
template <int BITS>
struct RowBits {
  static constexpr int kWords = (BITS * 32 + 31) / 32;
  uint32_t w[kWords + 1];
  __device__ __forceinline__ void load(const uint8_t *codes, int t, int cbase) {
    const int bitoff = BITS * (t * kDim + cbase);
    const uint32_t *p = reinterpret_cast<const uint32_t *>(codes) + (bitoff >> 5);
    const int sh = bitoff & 31;
    uint32_t raw[kWords + 2];
#pragma unroll
    for (int i = 0; i < kWords + 1; ++i) raw[i] = p[i];
    raw[kWords + 1] = 0;
#pragma unroll
    for (int i = 0; i < kWords + 1; ++i) w[i] = __funnelshift_r(raw[i], raw[i + 1], sh);
  }
  // x_j = 1 + code_j * 2^-BITS as a float: the code placed in the top BITS mantissa bits.
  __device__ __forceinline__ float x(int j) const {
    constexpr int kTop = 23 - BITS;
    const int pos = BITS * j, wi = pos >> 5, bi = pos & 31;
    uint32_t v;
    if (bi + BITS <= 32) {
      v = kTop >= bi ? (w[wi] << (kTop - bi)) : (w[wi] >> (bi - kTop));
    } else {
      v = __funnelshift_r(w[wi], w[wi + 1], bi) << kTop;
    }
    return __uint_as_float((v & (((1u << BITS) - 1u) << kTop)) | 0x3F800000u);
  }
};

// Restore rows t0 and t1 (this lane's 32 channels each) of a staged block and
// round them to the bridge dtype: out*[m] packs channels cbase+2m, cbase+2m+1.
template <int BITS, typename T>
__device__ __forceinline__ void restore_rows(const uint8_t *codes, const float *ma, const float *mb, int t0, int t1,
                                             int cbase, float n0, float n1, uint32_t (&out0)[16],
                                             uint32_t (&out1)[16]) {
  RowBits<BITS> r0, r1;
  r0.load(codes, t0, cbase);
  r1.load(codes, t1, cbase);
  float2 d0[16], d1[16];
  float2 ss0 = f2(0.f, 0.f), ss1 = f2(0.f, 0.f);
  const int mi = meta_index(cbase);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 a4 = *reinterpret_cast<const float4 *>(&ma[mi + 4 * q]);
    const float4 b4 = *reinterpret_cast<const float4 *>(&mb[mi + 4 * q]);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int m = 2 * q + e;
      const float2 a2 = e ? f2(a4.z, a4.w) : f2(a4.x, a4.y);
      const float2 b2 = e ? f2(b4.z, b4.w) : f2(b4.x, b4.y);
      d0[m] = __ffma2_rn(b2, f2(r0.x(2 * m), r0.x(2 * m + 1)), a2);
      d1[m] = __ffma2_rn(b2, f2(r1.x(2 * m), r1.x(2 * m + 1)), a2);
      ss0 = __ffma2_rn(d0[m], d0[m], ss0);
      ss1 = __ffma2_rn(d1[m], d1[m], ss1);
    }
  }
  float s0 = ss0.x + ss0.y, s1 = ss1.x + ss1.y;
  s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
  s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
  s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
  s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
  // norm / max(||d||, eps); the eps clamp only matters for an all-zero direction
  const float al0 = n0 == 0.f ? 0.f : (s0 > 1e-24f ? n0 * rsqrtf(s0) : n0 * 1e12f);
  const float al1 = n1 == 0.f ? 0.f : (s1 > 1e-24f ? n1 * rsqrtf(s1) : n1 * 1e12f);
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    out0[m] = pack2<T>(__fmul2_rn(d0[m], f2(al0, al0)));
    out1[m] = pack2<T>(__fmul2_rn(d1[m], f2(al1, al1)));
  }
}

// Scores of this warp's 16 tokens for the 8 query-head columns: D = K16 q^T.
template <typename T>
__device__ __forceinline__ void qk_mma(const uint32_t (&ka)[16], const uint32_t (&kb)[16], const uint32_t (&bq)[16],
                                       float (&d)[4]) {
  d[0] = d[1] = d[2] = d[3] = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t a[4] = {ka[2 * j], kb[2 * j], ka[2 * j + 1], kb[2 * j + 1]};
    mma16816<T>(d, a, bq[2 * j], bq[2 * j + 1]);
  }
}

// Write scores (D fragments) of rows t0, t1 for heads 2tig, 2tig+1 < G.
__device__ __forceinline__ void put_scores(float (&sc)[kHeads][kBlock], const float (&d)[4], int t0, int t1,
                                           int tig, int G, bool v0, bool v1) {
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int n = 2 * tig + e;
    if (n < G) {
      sc[n][t0] = v0 ? d[e] * kScale : -INFINITY;
      sc[n][t1] = v1 ? d[2 + e] * kScale : -INFINITY;
    }
  }
}

// Online softmax of one tile, per lane: lane (g, tig) owns query head g and the
// 16 tokens of its P.V B fragments (16ks + 2tig + {0,1,8,9}); the 4 lanes of a
// head cover all 64 tokens.  Returns the weights and rescales acc (heads 2tig,
// 2tig+1) to the new running max.  mrun/lrun are this lane's head-g state.
struct SoftState {
  float m = -INFINITY, l = 0.f;
};

__device__ __forceinline__ void softmax_lane(const float (&sc)[kHeads][kBlock], int g, int tig, int G,
                                             SoftState &ss, float (&p)[16], float (&acc)[2][4], int &st) {
  constexpr float kLog2e = 1.4426950408889634f;
  float bmax = -INFINITY;
  if (g < G) {
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const float2 a = *reinterpret_cast<const float2 *>(&sc[g][16 * ks + 2 * tig]);
      const float2 b = *reinterpret_cast<const float2 *>(&sc[g][16 * ks + 2 * tig + 8]);
      p[4 * ks] = a.x;
      p[4 * ks + 1] = a.y;
      p[4 * ks + 2] = b.x;
      p[4 * ks + 3] = b.y;
      bmax = fmaxf(bmax, fmaxf(fmaxf(a.x, a.y), fmaxf(b.x, b.y)));
    }
  }
  bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 1));
  bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 2));
  const float mnew = fmaxf(ss.m, bmax);
  float r = 1.f, psum = 0.f;
  if (g < G && mnew != -INFINITY) {
    r = exp2f((ss.m - mnew) * kLog2e);
    const float mb = mnew * kLog2e;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      p[i] = exp2f(fmaf(p[i], kLog2e, -mb));
      psum += p[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) p[i] = 0.f;
  }
  if (!isfinite(bmax) && bmax != -INFINITY) st |= NSNKV_ST_OUTPUT_NONFINITE;
  psum += __shfl_xor_sync(0xffffffffu, psum, 1);
  psum += __shfl_xor_sync(0xffffffffu, psum, 2);
  ss.l = ss.l * r + psum;
  ss.m = mnew;
  // rescale factors of the accumulator columns (heads 2tig, 2tig+1) from their owners
  const float r0 = __shfl_sync(0xffffffffu, r, 8 * tig);
  const float r1 = __shfl_sync(0xffffffffu, r, 8 * tig + 4);
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    acc[mt][0] *= r0;
    acc[mt][1] *= r1;
    acc[mt][2] *= r0;
    acc[mt][3] *= r1;
  }
}

// acc[mt] += V^T P for this warp's two 16-channel tiles over the 64 tokens of the tile.
template <typename T>
__device__ __forceinline__ void pv_mma(const uint16_t (*v16)[kVRow], const float (&p)[16], int warp, int lane,
                                       float (&acc)[2][4]) {
  const int mi = lane >> 3, r = lane & 7;
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const float2 pa = f2(p[4 * ks], p[4 * ks + 1]);
    const float2 pb = f2(p[4 * ks + 2], p[4 * ks + 3]);
    const uint32_t bhi0 = pack2<T>(pa), bhi1 = pack2<T>(pb);
    const float2 ha = unpack2<T>(bhi0), hb = unpack2<T>(bhi1);
    const uint32_t blo0 = pack2<T>(f2(pa.x - ha.x, pa.y - ha.y));
    const uint32_t blo1 = pack2<T>(f2(pb.x - hb.x, pb.y - hb.y));
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const int cm = 32 * warp + 16 * mt;
      uint32_t a[4];
      ldmatrix_x4_trans(a, &v16[16 * ks + r + 8 * (mi >> 1)][cm + 8 * (mi & 1)]);
      mma16816<T>(acc[mt], a, bhi0, bhi1);
      mma16816<T>(acc[mt], a, blo0, blo1);
    }
  }
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
__global__ void __launch_bounds__(kThreads, 4) attn_partial_kernel(const AttnArgs a) {
  constexpr int CB = code_bytes(BITS);
  constexpr float kTwoB = static_cast<float>(1 << BITS);
  extern __shared__ __align__(128) uint8_t smem_raw[];
  AttnSmem<BITS> &S = *reinterpret_cast<AttnSmem<BITS> *>(smem_raw);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tig = lane & 3, cbase = 32 * tig;
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
  // B fragments of q: column n = g is query head h*G + g (zero when g >= G).
  uint32_t bq[16];
  if (g < G) {
    load_row32<T>(static_cast<const T *>(a.q) + ((b * a.hq) + h * G + g) * kDim, cbase, bq);
    st |= check_row32<T>(bq);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) bq[i] = 0u;
  }
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  SoftState sm;
  float p[16];

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
    }
    __syncthreads();
    if (tid == 0)
      for (int i = 0; i < kStages && i < nloc; ++i) issue(blk0 + i, i);
    for (int li = 0; li < nloc; ++li) {
      const int s = li % kStages;
      const bool ok = mbar_wait_bounded(&S.full[s], (li / kStages) & 1, a.status);
      if (__syncthreads_or(!ok)) {
        // A staged copy never landed: give the later copies a bounded chance to
        // finish, then leave; the timeout status tells the host.
        if (tid == 0)
          for (int k = li + 1; k < nloc && k < li + kStages; ++k)
            mbar_wait_bounded(&S.full[k % kStages], (k / kStages) & 1, a.status);
        return;
      }
      const Stage<BITS> &sg = S.stage[s];
      MetaF &mf = S.meta[li & 1];
      {  // metadata of this block -> fp32 (a, b) pairs, one channel per thread
        const int c = tid, ci = meta_index(c);
        const float km = half_bits_to_f(sg.km[c]), ks = half_bits_to_f(sg.ks[c]);
        const float vm = half_bits_to_f(sg.vm[c]), vs = half_bits_to_f(sg.vs[c]);
        const float kb = ks * kTwoB, vb = vs * kTwoB;
        mf.ka[ci] = km - kb;
        mf.kb[ci] = kb;
        mf.va[ci] = vm - vb;
        mf.vb[ci] = vb;
        bool bad = !isfinite(km) || !isfinite(ks) || !isfinite(vm) || !isfinite(vs);
        if (c < kBlock) bad |= !isfinite(half_bits_to_f(sg.kn[c])) || !isfinite(half_bits_to_f(sg.vn[c]));
        if (bad) st |= NSNKV_ST_INPUT_NONFINITE;
      }
      __syncthreads();
      {
        uint32_t ka[16], kb[16];
        restore_rows<BITS, T>(sg.kc, mf.ka, mf.kb, t0, t1, cbase, half_bits_to_f(sg.kn[t0]),
                              half_bits_to_f(sg.kn[t1]), ka, kb);
        float d[4];
        qk_mma<T>(ka, kb, bq, d);
        put_scores(S.sc, d, t0, t1, tig, G, true, true);
        restore_rows<BITS, T>(sg.vc, mf.va, mf.vb, t0, t1, cbase, half_bits_to_f(sg.vn[t0]),
                              half_bits_to_f(sg.vn[t1]), ka, kb);
        store_row32(&S.v16[t0][cbase], ka);
        store_row32(&S.v16[t1][cbase], kb);
      }
      __syncthreads();
      // stage s is consumed: refill it with block li + kStages
      if (tid == 0 && li + kStages < nloc) issue(blk0 + li + kStages, s);
      softmax_lane(S.sc, g, tig, G, sm, p, acc, st);
      pv_mma<T>(S.v16, p, warp, lane, acc);
    }
  } else {
    // ---- native rows (tail, appended token, or materialised K/V), 64-token tiles
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
      if (tile > 0) __syncthreads();  // previous tile's P.V has finished reading sc / v16
      float d[4];
      qk_mma<T>(ka, kb, bq, d);
      put_scores(S.sc, d, t0, t1, tig, G, v0, v1);
      store_row32(&S.v16[t0][cbase], va);
      store_row32(&S.v16[t1][cbase], vb);
      __syncthreads();
      softmax_lane(S.sc, g, tig, G, sm, p, acc, st);
      pv_mma<T>(S.v16, p, warp, lane, acc);
    }
  }

  // ---- partial of this chunk: acc holds channels 32w + 16mt + {g, g+8}, heads 2tig, 2tig+1
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int n = 2 * tig + e;
    if (n < G) {
      const int64_t row = (b * a.hq + h * G + n) * a.max_chunks + chunk;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const int c = 32 * warp + 16 * mt + g;
        a.part_o[row * kDim + c] = acc[mt][e];
        a.part_o[row * kDim + c + 8] = acc[mt][2 + e];
      }
    }
  }
  if (warp == 0 && tig == 0 && g < G) {
    const int64_t row = (b * a.hq + h * G + g) * a.max_chunks + chunk;
    a.part_ml[row * 2] = sm.m;
    a.part_ml[row * 2 + 1] = sm.l;
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
