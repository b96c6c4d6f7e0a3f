// NSN block codec for sm_100a: encoder, restore (bridge reconstruct), bit pack/unpack,
// and the paged-cache seal.  All arithmetic that the reference performs on the CPU is
// reproduced bit for bit: every multiply/add/divide is individually rounded (no FMA
// contraction), square roots and divisions are IEEE, rounding is half-to-even, and the
// per-token sum of squares follows torch's CPU reduction order (nsnkv_common.cuh).
#include <type_traits>

#include "nsnkv_common.cuh"

namespace nsnkv {

// Shared-memory workspace of one 64x128 block encode/decode.
struct BlockSmem {
  float x[kBlock][kDim + 1];  // +1 pad: row-parallel reads are bank-conflict free
  float tok[kBlock];          // per-token norm (encode) or denominator (decode)
  float chan_min[kDim];
  float chan_scale[kDim];
  uint8_t q[kBlock * kDim];
  uint8_t packed[kBlock * kDim * 5 / 8];
};

// Running channel minimum in token order with torch's CPU tie rule: of equal values the
// later one is kept, so the minimum of a channel whose smallest value is zero carries the
// sign of its last zero (+0 and -0 compare equal; the sign reaches the fp16 min meta).
__device__ __forceinline__ float min_keep_last(float acc, float v) { return acc < v ? acc : v; }

template <typename T> __device__ __forceinline__ float load_elem(const T *p) { return Elem<T>::to_f(*p); }

// Load one contiguous 64x128 block into s.x (as float), flag non-finite input.
template <typename T>
__device__ __forceinline__ int load_block(const T *src, BlockSmem &s) {
  int bad = 0;
  constexpr int kVec = 16 / sizeof(T);  // elements per 16-byte load
  constexpr int kChunks = kBlock * kDim / kVec;
  for (int k = threadIdx.x; k < kChunks; k += blockDim.x) {
    int e = k * kVec;
    int r = e / kDim, c = e % kDim;
    uint4 raw = reinterpret_cast<const uint4 *>(src)[k];
    const T *v = reinterpret_cast<const T *>(&raw);
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
      float f = Elem<T>::to_f(v[j]);
      bad |= !isfinite(f);
      s.x[r][c + j] = f;
    }
  }
  return bad ? NSNKV_ST_INPUT_NONFINITE : 0;
}

// Pack s.q (8192 codes) into s.packed as the LSB-first bitstream.
template <int BITS>
__device__ __forceinline__ void pack_block(BlockSmem &s) {
  for (int g = threadIdx.x; g < kBlock * kDim / 8; g += blockDim.x) {
    const uint2 w = reinterpret_cast<const uint2 *>(s.q)[g];
    uint64_t v = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint32_t code = ((j < 4 ? w.x : w.y) >> (8 * (j & 3))) & 0xFFu;
      v |= static_cast<uint64_t>(code) << (BITS * j);
    }
#pragma unroll
    for (int b = 0; b < BITS; ++b) s.packed[g * BITS + b] = static_cast<uint8_t>(v >> (8 * b));
  }
}

// Encode the block held in s.x.  Outputs go to global memory (any may be null).
// Mirrors nsn_encode (loop_kv_nb06_primitives.py:37-55) step for step.
template <int BITS>
__device__ void encode_in_smem(BlockSmem &s, int norm_order, uint8_t *codes, int order, uint8_t *q_out,
                               uint16_t *norm, uint16_t *mn, uint16_t *scale, int32_t *status, int in_status) {
  const int tid = threadIdx.x;
  constexpr float kLevels = static_cast<float>((1 << BITS) - 1);
  int st = in_status;
  // n = ||x||_2 per token, torch's CPU order.
  if (tid < kBlock) {
    float ss = norm_order == 0 ? sumsq_lanes8(&s.x[tid][0], 1) : sumsq_seq(&s.x[tid][0], 1);
    float n = sqrtf(ss);
    s.tok[tid] = n;
    __half n16 = __float2half_rn(n);
    float n16f = __half2float(n16);
    if (!isfinite(n16f)) st |= NSNKV_ST_META_OVERFLOW;
    if (n != 0.f && n16f == 0.f) st |= NSNKV_ST_META_UNDERFLOW;
    if (norm) norm[tid] = __half_as_ushort(n16);
  }
  __syncthreads();
  // d = x / max(n, eps)
  for (int e = tid; e < kBlock * kDim; e += blockDim.x) {
    int r = e / kDim, c = e % kDim;
    s.x[r][c] = div_rn(s.x[r][c], fmaxf(s.tok[r], kEps));
  }
  __syncthreads();
  // per-channel min / scale, then codes
  for (int c = tid; c < kDim; c += blockDim.x) {
    float lo = s.x[0][c], hi = s.x[0][c];
    for (int r = 1; r < kBlock; ++r) {
      lo = min_keep_last(lo, s.x[r][c]);
      hi = fmaxf(hi, s.x[r][c]);
    }
    float sc = div_rn(sub_rn(hi, lo), kLevels);
    float denom = sc == 0.f ? 1.f : sc;
    for (int r = 0; r < kBlock; ++r) {
      float v = rintf(div_rn(sub_rn(s.x[r][c], lo), denom));
      v = fminf(fmaxf(v, 0.f), kLevels);
      uint8_t code = sc == 0.f ? 0 : static_cast<uint8_t>(v);
      s.q[r * kDim + c] = code;
    }
    __half m16 = __float2half_rn(lo), s16 = __float2half_rn(sc);
    float m16f = __half2float(m16), s16f = __half2float(s16);
    if (!isfinite(m16f) || !isfinite(s16f)) st |= NSNKV_ST_META_OVERFLOW;
    if (sc != 0.f && s16f == 0.f) st |= NSNKV_ST_META_UNDERFLOW;
    if (mn) mn[c] = __half_as_ushort(m16);
    if (scale) scale[c] = __half_as_ushort(s16);
  }
  __syncthreads();
  if (q_out) {
    for (int k = tid; k < kBlock * kDim / 16; k += blockDim.x)
      reinterpret_cast<uint4 *>(q_out)[k] = reinterpret_cast<const uint4 *>(s.q)[k];
  }
  if (codes) {
    pack_block<BITS>(s);
    __syncthreads();
    const uint16_t *h16 = reinterpret_cast<const uint16_t *>(s.packed);
    if (order == 1) {  // paired rows: word j*8*BITS + k = [row 2j half k | row 2j+1 half k]
      for (int w = tid; w < code_bytes(BITS) / 4; w += blockDim.x) {
        const int j = w / (8 * BITS), k = w % (8 * BITS);
        reinterpret_cast<uint32_t *>(codes)[w] =
            h16[2 * j * 8 * BITS + k] | (static_cast<uint32_t>(h16[(2 * j + 1) * 8 * BITS + k]) << 16);
      }
    } else if (order == 2) {  // paired halves: group word m = [A half m | B half m]
      for (int w = tid; w < code_bytes(BITS) / 4; w += blockDim.x) {
        const int grp = w / BITS, m = w % BITS;  // a 32-code group is BITS words
        reinterpret_cast<uint32_t *>(codes)[w] =
            h16[2 * BITS * grp + m] | (static_cast<uint32_t>(h16[2 * BITS * grp + BITS + m]) << 16);
      }
    } else {
      for (int k = tid; k < code_bytes(BITS) / 16; k += blockDim.x)
        reinterpret_cast<uint4 *>(codes)[k] = reinterpret_cast<const uint4 *>(s.packed)[k];
    }
  }
  if (st) set_status(status, st);
}

// ----------------------------------------------------------------- fp16 block encoder
// The same encode as encode_in_smem with every thread busy in every phase: a 64x128
// fp16 block is staged once in shared memory as fp32, each per-token and per-channel
// divisor gets one correctly rounded reciprocal, and the quotients of its elements
// are formed by quotient correction instead of a full IEEE division each:
//
//   y = RN(1/b),  q = RN(a*y),  then twice  q = RN(q + RN(a - b*q)*y)   (a - b*q by FMA)
//
// (Markstein's correction step, P. Markstein, "IA-64 and Elementary Functions",
// Prentice Hall 2000, ch. 8: with y within half an ulp of 1/b and q within one ulp
// of a/b, one correction gives the correctly rounded a/b; the first correction brings
// RN(a*y) within that ulp).  The argument needs every intermediate in the normal
// range, which holds for the fp16 encoder's operands: directions divide |x| <= 65504
// by b in [1e-12, 128^0.5 * 65504], codes divide d - min in [0, 2] by a scale that is
// either 1 or at least ~1e-22.  bf16 and fp32 inputs, whose range breaks that
// argument, keep the IEEE-division encoder above.
//
// Directions are formed negated, nd = x / (-b): with a negative divisor the
// corrections keep the sign of a zero quotient (x / b of -0 is -0, and the
// correction's "+ RN(a - b*q)*y" would otherwise turn -0 into +0).  min d = -max nd and
// max d = -min nd exactly.
constexpr int kXRowF = kDim + 8;  // fp32 words per staged row; the pad makes the norm phase's reads conflict-free

struct FastSmem {
  float x[kBlock][kXRowF];   // the block as fp32
  float nyt[kBlock];         // -RN(1 / max(n, eps)) per token
  float bt[kBlock];          // max(n, eps) per token
  float2 pmax[4][kDim / 2];  // per channel pair and token quarter: max of nd (= -min d) ...
  float2 pmin[4][kDim / 2];  // ... and min of nd (= -max d)
  uint8_t q[kBlock * kDim];  // codes, row-major (token, channel)
};

struct Recip2 {
  float2 y;   // RN(1/b) per lane
  float2 nb;  // -b per lane
};

__device__ __forceinline__ float2 div2_by(float2 a, const Recip2 &r) {
  float2 q = __fmul2_rn(a, r.y);
  float2 e = __ffma2_rn(q, r.nb, a);
  q = __ffma2_rn(e, r.y, q);
  e = __ffma2_rn(q, r.nb, a);
  return __ffma2_rn(e, r.y, q);
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float min3(float a, float b, float c) {
  float r;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 32 consecutive codes (one per byte of w) -> BITS words of the LSB-first bitstream.
template <int BITS>
__device__ __forceinline__ void pack32(const uint32_t (&w)[8], uint32_t (&out)[BITS]) {
  constexpr uint32_t m = (1u << BITS) - 1u;
  constexpr uint32_t kM1 = m * 0x00010001u;             // codes of bytes 0 and 2 in place
  constexpr uint32_t kM2 = (m << BITS) * 0x00010001u;   // codes of bytes 1 and 3 moved down next to them
  constexpr uint32_t kF = (1u << (2 * BITS)) - 1u;
  uint64_t acc = 0;
  int nbits = 0, o = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t p = (w[k] & kM1) | ((w[k] >> (8 - BITS)) & kM2);
    const uint32_t f = (p & kF) | ((p >> (16 - 2 * BITS)) & (kF << (2 * BITS)));
    acc |= static_cast<uint64_t>(f) << nbits;
    nbits += 4 * BITS;
    if (nbits >= 32) {
      out[o++] = static_cast<uint32_t>(acc);
      acc >>= 32;
      nbits -= 32;
    }
  }
}

// Encode one contiguous 64x128 fp16 block (256 threads).  Outputs as encode_in_smem;
// codes and q_out may be null.
// Stage one contiguous 64x128 fp16 block into s.x as fp32 (all 256 threads).  Thread k
// of a row's 16 writes its 32 bytes as two 16-byte halves, the second half first on
// odd-numbered quarters of the row, so each quarter-warp store covers all 32 banks.
__device__ __forceinline__ void stage_block(const __half *src, FastSmem &s) {
  const uint4 *g = reinterpret_cast<const uint4 *>(src);
  uint4 v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = g[threadIdx.x + 256 * j];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int k = threadIdx.x + 256 * j;
    float *dst = &s.x[k >> 4][(k & 15) * 8];
    const float2 a = Elem<__half>::to_f2(v[j].x), b = Elem<__half>::to_f2(v[j].y);
    const float2 c = Elem<__half>::to_f2(v[j].z), d = Elem<__half>::to_f2(v[j].w);
    const float4 lo = make_float4(a.x, a.y, b.x, b.y), hi = make_float4(c.x, c.y, d.x, d.y);
    const int swap = (k >> 2) & 1;
    *reinterpret_cast<float4 *>(dst + 4 * swap) = swap ? hi : lo;
    *reinterpret_cast<float4 *>(dst + 4 * (swap ^ 1)) = swap ? lo : hi;
  }
}

template <int BITS>
__device__ void encode_block_fast(const __half *src, uint8_t *codes, int order, uint8_t *q_out, uint16_t *norm,
                                  uint16_t *mn,
                                  uint16_t *scale, int32_t *status, FastSmem &s) {
  const int t = threadIdx.x;
  constexpr uint32_t kL = (1u << BITS) - 1u;
  int st = 0;
  stage_block(src, s);
  __syncthreads();
  // n = ||x||_2 per token in torch's CPU order: thread (r, g) runs lanes 2g and 2g+1
  // of the eight interleaved accumulators, then the lanes are added 0..7.
  {
    const int r = t >> 2, g = t & 3;
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float2 v = *reinterpret_cast<const float2 *>(&s.x[r][8 * k + 2 * g]);
      const float2 sq = __fmul2_rn(v, v);
      acc = k == 0 ? sq : __fadd2_rn(acc, sq);
    }
    const int base = t & 28;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lx = __shfl_sync(0xffffffffu, acc.x, base + j);
      const float ly = __shfl_sync(0xffffffffu, acc.y, base + j);
      ss = j == 0 ? add_rn(lx, ly) : add_rn(add_rn(ss, lx), ly);
    }
    // |x| <= 65504 keeps 128 squares finite: a non-finite sum means a non-finite input
    if (!isfinite(ss)) st |= NSNKV_ST_INPUT_NONFINITE;
    if (g == 0) {
      const float n = __fsqrt_rn(ss);
      const float b = fmaxf(n, kEps);
      s.bt[r] = b;
      s.nyt[r] = -__frcp_rn(b);
      const __half n16 = __float2half_rn(n);
      const float n16f = __half2float(n16);
      if (!isfinite(n16f)) st |= NSNKV_ST_META_OVERFLOW;
      if (n != 0.f && n16f == 0.f) st |= NSNKV_ST_META_UNDERFLOW;
      norm[r] = __half_as_ushort(n16);
    }
  }
  __syncthreads();
  // nd = x / -max(n, eps) for channel pair cp over token quarter tg, with its max / min
  const int cp = t & 63, tg = t >> 6;
  float2 nd[16];
  float2 mx = make_float2(-INFINITY, -INFINITY), mnv = make_float2(INFINITY, INFINITY);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 ny4 = *reinterpret_cast<const float4 *>(&s.nyt[16 * tg + 4 * j]);
    const float4 b4 = *reinterpret_cast<const float4 *>(&s.bt[16 * tg + 4 * j]);
    const float nyv[4] = {ny4.x, ny4.y, ny4.z, ny4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = 4 * j + e;
      const float2 v = *reinterpret_cast<const float2 *>(&s.x[16 * tg + i][2 * cp]);
      nd[i] = div2_by(v, Recip2{make_float2(nyv[e], nyv[e]), make_float2(bv[e], bv[e])});
    }
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const int i = 4 * j + e;
      mx = make_float2(max3(mx.x, nd[i].x, nd[i + 1].x), max3(mx.y, nd[i].y, nd[i + 1].y));
      mnv = make_float2(min3(mnv.x, nd[i].x, nd[i + 1].x), min3(mnv.y, nd[i].y, nd[i + 1].y));
    }
  }
  s.pmax[tg][cp] = mx;
  s.pmin[tg][cp] = mnv;
  __syncthreads();
  {
    const float2 a0 = s.pmax[0][cp], a1 = s.pmax[1][cp], a2 = s.pmax[2][cp], a3 = s.pmax[3][cp];
    const float2 b0 = s.pmin[0][cp], b1 = s.pmin[1][cp], b2 = s.pmin[2][cp], b3 = s.pmin[3][cp];
    mx = make_float2(max3(a0.x, a1.x, fmaxf(a2.x, a3.x)), max3(a0.y, a1.y, fmaxf(a2.y, a3.y)));
    mnv = make_float2(min3(b0.x, b1.x, fminf(b2.x, b3.x)), min3(b0.y, b1.y, fminf(b2.y, b3.y)));
  }
  // channel min / max of d; a zero min gets its sign fixed below
  const float2 lo = make_float2(-mx.x, -mx.y), hi = make_float2(-mnv.x, -mnv.y);
  const float scx = div_rn(sub_rn(hi.x, lo.x), static_cast<float>(kL));
  const float scy = div_rn(sub_rn(hi.y, lo.y), static_cast<float>(kL));
  const float dx = scx == 0.f ? 1.f : scx, dy = scy == 0.f ? 1.f : scy;
  if (tg == 0) {
    const __half2 m16 = __floats2half2_rn(lo.x, lo.y), s16 = __floats2half2_rn(scx, scy);
    const float2 m16f = __half22float2(m16), s16f = __half22float2(s16);
    if (!isfinite(m16f.x) || !isfinite(m16f.y) || !isfinite(s16f.x) || !isfinite(s16f.y))
      st |= NSNKV_ST_META_OVERFLOW;
    if ((scx != 0.f && s16f.x == 0.f) || (scy != 0.f && s16f.y == 0.f)) st |= NSNKV_ST_META_UNDERFLOW;
    *reinterpret_cast<__half2 *>(mn + 2 * cp) = m16;
    *reinterpret_cast<__half2 *>(scale + 2 * cp) = s16;
  }
  // codes: rint((d - min) / scale), d - min = RN(max nd - nd) >= 0.  Adding 1.5 * 2^23
  // rounds the quotient (at most L * (1 + 2^-23)) to the nearest integer, ties to
  // even, into the low mantissa byte.  A channel whose scale is 0 divides by 1 values
  // below 2^-126 * 31: its codes are 0.
  {
    const Recip2 rc{make_float2(__frcp_rn(dx), __frcp_rn(dy)), make_float2(-dx, -dy)};
    const float2 magic = make_float2(12582912.f, 12582912.f);
    const float2 neg1 = make_float2(-1.f, -1.f);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float2 w = __fadd2_rn(div2_by(__ffma2_rn(nd[i], neg1, mx), rc), magic);
      const uint32_t pair = __byte_perm(__float_as_uint(w.x), __float_as_uint(w.y), 0x0040);
      *reinterpret_cast<uint16_t *>(&s.q[(16 * tg + i) * kDim + 2 * cp]) = static_cast<uint16_t>(pair);
    }
  }
  // torch keeps the later of equal values in its channel min, so a zero min carries the
  // sign of the channel's last zero in token order (rare: only channels without negatives)
  const int zero_min = tg == 0 && (lo.x == 0.f || lo.y == 0.f);
  if (__syncthreads_or(zero_min)) {
    uint32_t z = 0;  // per channel: 0 no zero, 1 last zero is +0, 2 last zero is -0 (of d = -nd)
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (nd[i].x == 0.f) z = (z & ~3u) | (signbit(nd[i].x) ? 1u : 2u);
      if (nd[i].y == 0.f) z = (z & ~12u) | ((signbit(nd[i].y) ? 1u : 2u) << 2);
    }
    reinterpret_cast<uint32_t *>(&s.pmax[0][0])[tg * (kDim / 2) + cp] = z;
    __syncthreads();
    if (zero_min) {
      uint16_t *m = mn + 2 * cp;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        if ((c == 0 ? lo.x : lo.y) != 0.f) continue;
        uint32_t last = 0;
        for (int j = 0; j < 4; ++j) {
          const uint32_t zj = (reinterpret_cast<const uint32_t *>(&s.pmax[0][0])[j * (kDim / 2) + cp] >> (2 * c)) & 3u;
          if (zj) last = zj;
        }
        m[c] = last == 2 ? 0x8000u : 0x0000u;
      }
    }
  }
  {
    const uint4 a = reinterpret_cast<const uint4 *>(s.q)[2 * t];
    const uint4 b = reinterpret_cast<const uint4 *>(s.q)[2 * t + 1];
    if (q_out) {
      reinterpret_cast<uint4 *>(q_out)[2 * t] = a;
      reinterpret_cast<uint4 *>(q_out)[2 * t + 1] = b;
    }
    if (codes) {
      const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      uint32_t out[BITS];
      pack32<BITS>(w, out);
      if (order == 1) {
        // thread t holds words BITS*(t&3).. of row t>>2; thread t^4 the same words of the other row
        // of the pair.  Pair word j*8*BITS + k = [row 2j half k | row 2j+1 half k]: the even row's
        // thread writes the even k, the odd row's thread the odd k.
        const bool odd = (t >> 2) & 1;
        uint32_t *dst = reinterpret_cast<uint32_t *>(codes) + (t >> 3) * 8 * BITS + 2 * BITS * (t & 3) + (odd ? 1 : 0);
#pragma unroll
        for (int i = 0; i < BITS; ++i) {
          const uint32_t other = __shfl_xor_sync(0xffffffffu, out[i], 4);
          dst[2 * i] = odd ? __byte_perm(other, out[i], 0x7632) : __byte_perm(out[i], other, 0x5410);
        }
      } else if (order == 2) {
        // thread t holds exactly one 32-code group (2*BITS halves, half k in word k/2):
        // word m = [half m | half BITS+m]
        uint32_t *dst = reinterpret_cast<uint32_t *>(codes) + BITS * t;
#pragma unroll
        for (int m = 0; m < BITS; ++m) {
          const int ka = m, kb = BITS + m;
          const uint32_t sel = ((ka & 1) ? 0x0032u : 0x0010u) | ((kb & 1) ? 0x7600u : 0x5400u);
          dst[m] = __byte_perm(out[ka >> 1], out[kb >> 1], sel);
        }
      } else {
        uint32_t *dst = reinterpret_cast<uint32_t *>(codes) + BITS * t;
#pragma unroll
        for (int i = 0; i < BITS; ++i) dst[i] = out[i];
      }
    }
  }
  if (st) set_status(status, st);
}

__device__ __forceinline__ void write_header(uint8_t *h, int64_t offset, int bits) {
  uint64_t off = static_cast<uint64_t>(offset);
#pragma unroll
  for (int b = 0; b < 8; ++b) h[b] = static_cast<uint8_t>(off >> (8 * b));
  h[8] = kBlock & 0xFF;
  h[9] = kBlock >> 8;
  h[10] = static_cast<uint8_t>(bits);
  h[11] = 0;
}

// Input block b = r*blocks_per_row + i is written to output block index
// r*out_row_stride + out_offset + i (a contiguous [rows][blocks_per_row] layout when
// out_row_stride == blocks_per_row and out_offset == 0; a head-major page pool otherwise).
template <typename T, int BITS>
__global__ void __launch_bounds__(256) encode_blocks_kernel(const T *x, int norm_order, int64_t blocks_per_row,
                                                            uint8_t *codes, uint8_t *q_out, uint16_t *norm,
                                                            uint16_t *mn, uint16_t *scale, uint8_t *headers,
                                                            int64_t header_start, int64_t out_row_stride,
                                                            int64_t out_offset, int64_t cs, int64_t ms, int order,
                                                            int32_t *status) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  BlockSmem &s = *reinterpret_cast<BlockSmem *>(smem_raw);
  const int64_t b = blockIdx.x;
  const int64_t r = b / blocks_per_row, i = b % blocks_per_row;
  const int64_t o = r * out_row_stride + out_offset + i;
  int st = load_block<T>(x + b * kBlock * kDim, s);
  __syncthreads();
  encode_in_smem<BITS>(s, norm_order, codes ? codes + o * cs : nullptr, order,
                       q_out ? q_out + b * kBlock * kDim : nullptr,
                       norm + o * kBlock, blk_ptr(mn, o, ms), blk_ptr(scale, o, ms), status, st);
  if (headers && threadIdx.x == 0) write_header(headers + o * 12, header_start + kBlock * i, BITS);
}

template <int BITS>
__global__ void __launch_bounds__(256, 4) encode_blocks_fast_kernel(const __half *x, int64_t blocks_per_row,
                                                                   uint8_t *codes, uint8_t *q_out, uint16_t *norm,
                                                                   uint16_t *mn, uint16_t *scale, uint8_t *headers,
                                                                   int64_t header_start, int64_t out_row_stride,
                                                                   int64_t out_offset, int64_t cs, int64_t ms,
                                                                   int order, int32_t *status) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  FastSmem &s = *reinterpret_cast<FastSmem *>(smem_raw);
  const int64_t b = blockIdx.x;
  const int64_t r = b / blocks_per_row, i = b % blocks_per_row;
  const int64_t o = r * out_row_stride + out_offset + i;
  encode_block_fast<BITS>(x + b * kBlock * kDim, codes ? codes + o * cs : nullptr, order,
                          q_out ? q_out + b * kBlock * kDim : nullptr, norm + o * kBlock, blk_ptr(mn, o, ms),
                          blk_ptr(scale, o, ms), status, s);
  if (headers && threadIdx.x == 0) write_header(headers + o * 12, header_start + kBlock * i, BITS);
}

// ----------------------------------------------------------------- restore
// d = m + s*q (separately rounded), y = n * (d / max(||d||, eps)), 0 where n == 0.
// Mirrors nsn_decode (loop_kv_nb06_primitives.py:57-66).
template <typename T, int BITS>
__global__ void __launch_bounds__(256) restore_kernel(const uint8_t *codes, int codes_unpacked, const uint16_t *norm,
                                                      const uint16_t *mn, const uint16_t *scale,
                                                      int64_t blocks_per_row, int64_t row_tokens, T *out,
                                                      int32_t *status) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  BlockSmem &s = *reinterpret_cast<BlockSmem *>(smem_raw);
  const int64_t b = blockIdx.x;
  const int tid = threadIdx.x;
  int st = 0;
  if (tid < kDim) {
    s.chan_min[tid] = half_bits_to_f(mn[b * kDim + tid]);
    s.chan_scale[tid] = half_bits_to_f(scale[b * kDim + tid]);
    if (!isfinite(s.chan_min[tid]) || !isfinite(s.chan_scale[tid])) st |= NSNKV_ST_INPUT_NONFINITE;
  }
  if (codes_unpacked) {
    const uint8_t *q = codes + b * kBlock * kDim;
    for (int k = tid; k < kBlock * kDim / 16; k += blockDim.x)
      reinterpret_cast<uint4 *>(s.q)[k] = reinterpret_cast<const uint4 *>(q)[k];
  } else {
    const uint8_t *src = codes + b * code_bytes(BITS);
    for (int k = tid; k < code_bytes(BITS) / 16; k += blockDim.x)
      reinterpret_cast<uint4 *>(s.packed)[k] = reinterpret_cast<const uint4 *>(src)[k];
  }
  __syncthreads();
  for (int e = tid; e < kBlock * kDim; e += blockDim.x) {
    uint32_t code;
    if (codes_unpacked) {
      code = s.q[e];
    } else {
      int pos = e * BITS;
      uint32_t lo = s.packed[pos >> 3];
      uint32_t hi = (pos >> 3) + 1 < code_bytes(BITS) ? s.packed[(pos >> 3) + 1] : 0u;
      code = ((lo | (hi << 8)) >> (pos & 7)) & ((1u << BITS) - 1u);
    }
    int r = e / kDim, c = e % kDim;
    s.x[r][c] = add_rn(s.chan_min[c], mul_rn(s.chan_scale[c], static_cast<float>(code)));
  }
  __syncthreads();
  if (tid < kBlock) {
    float ss = sumsq_lanes8(&s.x[tid][0], 1);
    s.tok[tid] = fmaxf(sqrtf(ss), kEps);
  }
  __syncthreads();
  const int64_t row = b / blocks_per_row, blk = b % blocks_per_row;
  T *dst = out + (row * row_tokens + blk * kBlock) * kDim;
  for (int e = tid; e < kBlock * kDim; e += blockDim.x) {
    int r = e / kDim, c = e % kDim;
    float n = half_bits_to_f(norm[b * kBlock + r]);
    float y = n == 0.f ? 0.f : mul_rn(n, div_rn(s.x[r][c], s.tok[r]));
    T o = Elem<T>::from_f(y);
    if (!isfinite(Elem<T>::to_f(o)) || !isfinite(n)) st |= (!isfinite(n) ? NSNKV_ST_INPUT_NONFINITE : NSNKV_ST_OUTPUT_NONFINITE);
    dst[e] = o;
  }
  if (st) set_status(status, st);
}

template <typename T>
__global__ void copy_tail_kernel(const T *tail, int64_t rows, int64_t tail_len, int64_t row_tokens, int64_t offset_tokens,
                                 T *out, int32_t *status) {
  const int64_t n = rows * tail_len * kDim;
  int bad = 0;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t r = e / (tail_len * kDim), rem = e % (tail_len * kDim);
    T v = tail[e];
    bad |= !isfinite(Elem<T>::to_f(v));
    out[r * row_tokens * kDim + offset_tokens * kDim + rem] = v;
  }
  if (bad) set_status(status, NSNKV_ST_INPUT_NONFINITE);
}

// ----------------------------------------------------------------- bitstream pack / unpack
__global__ void pack_kernel(const uint8_t *codes, int64_t count, int bits, uint8_t *out, int32_t *status) {
  const int64_t groups = (count + 7) / 8;
  const int64_t total = (count * bits + 7) / 8;
  int bad = 0;
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < groups;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint64_t v = 0;
    for (int j = 0; j < 8; ++j) {
      int64_t i = g * 8 + j;
      if (i < count) {
        uint32_t c = codes[i];
        bad |= c >> bits;
        v |= static_cast<uint64_t>(c & ((1u << bits) - 1u)) << (bits * j);
      }
    }
    for (int b = 0; b < bits; ++b) {
      int64_t o = g * bits + b;
      if (o < total) out[o] = static_cast<uint8_t>(v >> (8 * b));
    }
  }
  if (bad) set_status(status, NSNKV_ST_INPUT_NONFINITE);
}

__global__ void unpack_kernel(const uint8_t *payload, int64_t count, int bits, uint8_t *out) {
  const int64_t groups = (count + 7) / 8;
  const int64_t total = (count * bits + 7) / 8;
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < groups;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint64_t v = 0;
    for (int b = 0; b < bits; ++b) {
      int64_t o = g * bits + b;
      if (o < total) v |= static_cast<uint64_t>(payload[o]) << (8 * b);
    }
    for (int j = 0; j < 8; ++j) {
      int64_t i = g * 8 + j;
      if (i < count) out[i] = static_cast<uint8_t>((v >> (bits * j)) & ((1u << bits) - 1u));
    }
  }
}

// ----------------------------------------------------------------- paged-cache seal
template <int BITS>
__device__ void renorm_block(const uint8_t *codes, int order, const uint16_t *norm, const uint16_t *mn,
                             const uint16_t *sc, float *alpha);

// One CTA per (kv head, K|V, sequence).  A sequence whose tail holds 64 tokens has that
// tail encoded into its next page, and with k_alpha the page's renorm factors written
// by the same CTA.  With `done` (per-sequence counters, zero between calls) the CTA that
// finishes a sequence last also advances its n_blocks / tail_len and resets the counter,
// so no separate counter kernel runs; every CTA reads the counters before it counts.
template <typename T, int BITS>
__global__ void __launch_bounds__(256) seal_kernel(const T *k_tail, const T *v_tail, int64_t tss, int64_t tsh,
                                                   int32_t *tail_len, int32_t *n_blocks, int pending,
                                                   const int32_t *table, int64_t table_stride, uint8_t *k_codes,
                                                   uint16_t *k_norm, uint16_t *k_min, uint16_t *k_scale,
                                                   uint8_t *v_codes, uint16_t *v_norm, uint16_t *v_min,
                                                   uint16_t *v_scale, float *k_alpha, float *v_alpha, int32_t *done,
                                                   int64_t sh, int64_t sp, int64_t cs, int64_t ms, int rec_order,
                                                   int32_t *status) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  // launched with a programmatic dependency: wait for the kernel before it, then let the
  // next one (the following decode step) launch while this grid runs
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int h = blockIdx.x, kv = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int32_t tl = tail_len[b], nbk = n_blocks[b];
  // a full tail seals into page n_blocks[b] of the sequence's table row; with no page
  // left in the row it stays a full tail and the status says so (the next append is refused)
  const bool room = nbk < table_stride;
  const bool full = tl + pending >= kBlock && room;
  if (tl + pending >= kBlock && !room && h == 0 && kv == 0 && threadIdx.x == 0) set_status(status, NSNKV_ST_CAPACITY);
  if (!full && !done) return;
  if (full) {
    const int32_t page = table[b * table_stride + nbk];
    const int64_t blk = h * sh + static_cast<int64_t>(page) * sp;
    const T *src = (kv == 0 ? k_tail : v_tail) + (b * tss + h * tsh) * kDim;
    uint8_t *codes = (kv == 0 ? k_codes : v_codes) + blk * cs;
    uint16_t *nrm = (kv == 0 ? k_norm : v_norm) + blk * kBlock;
    uint16_t *mn = blk_ptr(kv == 0 ? k_min : v_min, blk, ms);
    uint16_t *sc = blk_ptr(kv == 0 ? k_scale : v_scale, blk, ms);
    const int order = rec_order ? (kv == 0 ? 2 : 1) : 0;  // the block records' K and V code orders
    if constexpr (std::is_same<T, __half>::value) {
      encode_block_fast<BITS>(src, codes, order, nullptr, nrm, mn, sc, status,
                              *reinterpret_cast<FastSmem *>(smem_raw));
    } else {
      BlockSmem &s = *reinterpret_cast<BlockSmem *>(smem_raw);
      int st = load_block<T>(src, s);
      __syncthreads();
      encode_in_smem<BITS>(s, 0, codes, order, nullptr, nrm, mn, sc, status, st);
    }
    if (k_alpha) {
      __syncthreads();  // this CTA's code and metadata stores are visible to all its threads
      renorm_block<BITS>(codes, order, nrm, mn, sc, blk_ptr(kv == 0 ? k_alpha : v_alpha, blk, ms));
    }
  }
  if (done) {
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      const int per_seq = static_cast<int>(gridDim.x * gridDim.y);
      if (atomicAdd(&done[b], 1) == per_seq - 1) {
        // a full tail without a page keeps its rows: an append to it was not stored
        const int64_t t = tl + pending;
        n_blocks[b] = nbk + (full ? 1 : 0);
        tail_len[b] = static_cast<int32_t>(full ? t - kBlock : (t < tsh ? t : tsh));
        done[b] = 0;
      }
    }
  }
}

__global__ void seal_update_kernel(int64_t batch, int32_t *tail_len, int32_t *n_blocks, int pending,
                                   int64_t table_stride, int64_t tail_rows) {
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b < batch;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int32_t t = tail_len[b] + pending;
    if (t > tail_rows) t = static_cast<int32_t>(tail_rows);  // an append to a full tail was not stored
    if (t >= kBlock && n_blocks[b] < table_stride) {  // (seal_kernel left a tail without a page full)
      n_blocks[b] += 1;
      t -= kBlock;
    }
    tail_len[b] = t;
  }
}

// ----------------------------------------------------------------- per-token renorm factors
// alpha_t = n_t / max(||d_t||, eps), and 0 when n_t == 0, with d = min + scale * code in
// fp32: the factor nsn_decode applies to a row (loop_kv_nb06_primitives.py:57-66,
// y = n * d / max(||d||, eps)).  Decode attention over a cache that stores it beside
// each block does not recompute ||d|| on every step.  One 256-thread CTA per block:
// thread (t = tid / 4, quarter) sums 32 channels of token t.
template <int BITS>
__device__ void renorm_block(const uint8_t *codes, int order, const uint16_t *norm, const uint16_t *mn,
                             const uint16_t *sc, float *alpha) {
  const int t = threadIdx.x >> 2, part = threadIdx.x & 3;
  constexpr int row_bytes = kDim * BITS / 8;
  float ss = 0.f;
  for (int c = 32 * part; c < 32 * part + 32; ++c) {
    const int bit = c * BITS;  // within token t's packed row
    const int byte = bit >> 3, sh = bit & 7;
    uint32_t w = codes[code_byte_at(t, byte, BITS, order)];
    if (sh + BITS > 8 && byte + 1 < row_bytes)
      w |= static_cast<uint32_t>(codes[code_byte_at(t, byte + 1, BITS, order)]) << 8;
    const float x = static_cast<float>((w >> sh) & ((1u << BITS) - 1u));
    const float d = __fadd_rn(half_bits_to_f(mn[c]), __fmul_rn(half_bits_to_f(sc[c]), x));
    ss = __fmaf_rn(d, d, ss);
  }
  ss += __shfl_xor_sync(0xffffffffu, ss, 1);
  ss += __shfl_xor_sync(0xffffffffu, ss, 2);
  if (part == 0) {
    const float n = half_bits_to_f(norm[t]);
    alpha[t] = n == 0.f ? 0.f : __fdiv_rn(n, fmaxf(__fsqrt_rn(ss), kEps));
  }
}

// Blocks laid out as nsnkv_encode_blocks writes them: block (row r, i) at r * row_stride + offset + i;
// consecutive blocks are cs bytes apart in codes and ms bytes apart in min / scale / alpha.
template <int BITS>
__global__ void __launch_bounds__(256) renorm_blocks_kernel(const uint8_t *codes, const uint16_t *norm,
                                                            const uint16_t *mn, const uint16_t *sc,
                                                            int64_t blocks_per_row, int64_t row_stride,
                                                            int64_t offset, float *alpha, int64_t cs, int64_t ms,
                                                            int order) {
  const int64_t r = blockIdx.x / blocks_per_row, i = blockIdx.x % blocks_per_row;
  const int64_t blk = r * row_stride + offset + i;
  renorm_block<BITS>(codes + blk * cs, order, norm + blk * kBlock, blk_ptr(mn, blk, ms),
                     blk_ptr(sc, blk, ms), blk_ptr(alpha, blk, ms));
}

// ----------------------------------------------------------------- host dispatch
template <typename T>
static int launch_encode(const void *x, int64_t n_blocks, int64_t bpr, int bits, int norm_order, uint8_t *codes,
                         uint8_t *q_out, uint16_t *norm, uint16_t *mn, uint16_t *scale, uint8_t *headers,
                         int64_t header_start, int64_t out_row_stride, int64_t out_offset, int64_t cs, int64_t ms,
                         int order, int32_t *status, cudaStream_t st) {
  dim3 grid(static_cast<unsigned>(n_blocks));
  if (std::is_same<T, __half>::value && norm_order == 0) {
    const size_t smem = sizeof(FastSmem);
#define NSNKV_ENC_FAST(B)                                                                                  \
  case B: {                                                                                                \
    auto k = encode_blocks_fast_kernel<B>;                                                                 \
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)        \
      return NSNKV_ERR_CUDA;                                                                               \
    k<<<grid, 256, smem, st>>>(static_cast<const __half *>(x), bpr, codes, q_out, norm, mn, scale, headers, \
                               header_start, out_row_stride, out_offset, cs, ms, order, status);           \
    break;                                                                                                 \
  }
    switch (bits) {
      NSNKV_ENC_FAST(3)
      NSNKV_ENC_FAST(4)
      NSNKV_ENC_FAST(5)
      default:
        return NSNKV_ERR_ARG;
    }
#undef NSNKV_ENC_FAST
    return cudaGetLastError() == cudaSuccess ? NSNKV_OK : NSNKV_ERR_LAUNCH;
  }
  const size_t smem = sizeof(BlockSmem);
#define NSNKV_ENC(B)                                                                                      \
  case B: {                                                                                               \
    auto k = encode_blocks_kernel<T, B>;                                                                  \
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)       \
      return NSNKV_ERR_CUDA;                                                                              \
    k<<<grid, 256, smem, st>>>(static_cast<const T *>(x), norm_order, bpr, codes, q_out, norm, mn, scale, \
                               headers, header_start, out_row_stride, out_offset, cs, ms, order, status);  \
    break;                                                                                                \
  }
  switch (bits) {
    NSNKV_ENC(3)
    NSNKV_ENC(4)
    NSNKV_ENC(5)
    default:
      return NSNKV_ERR_ARG;
  }
#undef NSNKV_ENC
  return cudaGetLastError() == cudaSuccess ? NSNKV_OK : NSNKV_ERR_LAUNCH;
}

template <typename T>
static int launch_restore(const uint8_t *codes, int unpacked, const uint16_t *norm, const uint16_t *mn,
                          const uint16_t *scale, int64_t rows, int64_t bpr, int bits, const void *tail,
                          int64_t tail_len, void *out, int32_t *status, cudaStream_t st) {
  const size_t smem = sizeof(BlockSmem);
  const int64_t row_tokens = bpr * kBlock + tail_len;
  const int64_t n = rows * bpr;
  if (n > 0) {
    dim3 grid(static_cast<unsigned>(n));
#define NSNKV_RES(B)                                                                                       \
  case B: {                                                                                                \
    auto k = restore_kernel<T, B>;                                                                         \
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)        \
      return NSNKV_ERR_CUDA;                                                                               \
    k<<<grid, 256, smem, st>>>(codes, unpacked, norm, mn, scale, bpr, row_tokens, static_cast<T *>(out),   \
                               status);                                                                    \
    break;                                                                                                 \
  }
    switch (bits) {
      NSNKV_RES(3)
      NSNKV_RES(4)
      NSNKV_RES(5)
      default:
        return NSNKV_ERR_ARG;
    }
#undef NSNKV_RES
  }
  if (tail_len > 0) {
    int64_t total = rows * tail_len * kDim;
    unsigned blocks = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 4096));
    copy_tail_kernel<T><<<blocks, 256, 0, st>>>(static_cast<const T *>(tail), rows, tail_len, row_tokens,
                                                bpr * kBlock, static_cast<T *>(out), status);
  }
  return cudaGetLastError() == cudaSuccess ? NSNKV_OK : NSNKV_ERR_LAUNCH;
}

template <typename T>
static int launch_seal(int64_t batch, int h, int bits, void *k_tail, void *v_tail, int64_t tss, int64_t tsh,
                       int32_t *tail_len, int32_t *n_blocks, int pending, const int32_t *table, int64_t ts,
                       uint8_t *kc, uint16_t *kn, uint16_t *km, uint16_t *ks, uint8_t *vc, uint16_t *vn,
                       uint16_t *vm, uint16_t *vs, float *ka, float *va, int32_t *done, int64_t sh, int64_t sp,
                       int64_t cs, int64_t ms, int rec_order, int32_t *status, cudaStream_t st) {
  const size_t smem = std::is_same<T, __half>::value ? sizeof(FastSmem) : sizeof(BlockSmem);
  dim3 grid(h, 2, static_cast<unsigned>(batch));
#define NSNKV_SEAL(B)                                                                                      \
  case B: {                                                                                                \
    auto k = seal_kernel<T, B>;                                                                            \
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)        \
      return NSNKV_ERR_CUDA;                                                                               \
    cudaLaunchConfig_t cfg{};                                                                              \
    cfg.gridDim = grid;                                                                                    \
    cfg.blockDim = dim3(256);                                                                              \
    cfg.dynamicSmemBytes = smem;                                                                           \
    cfg.stream = st;                                                                                       \
    cudaLaunchAttribute attr[1];                                                                           \
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;                                       \
    attr[0].val.programmaticStreamSerializationAllowed = 1;                                                \
    cfg.attrs = attr;                                                                                      \
    cfg.numAttrs = 1;                                                                                      \
    if (cudaLaunchKernelEx(&cfg, k, static_cast<const T *>(k_tail), static_cast<const T *>(v_tail), tss,   \
                           tsh, tail_len, n_blocks, pending, table, ts, kc, kn, km, ks, vc, vn, vm, vs, ka, \
                           va, done, sh, sp, cs, ms, rec_order, status) != cudaSuccess)                    \
      return NSNKV_ERR_LAUNCH;                                                                             \
    break;                                                                                                 \
  }
  switch (bits) {
    NSNKV_SEAL(3)
    NSNKV_SEAL(4)
    NSNKV_SEAL(5)
    default:
      return NSNKV_ERR_ARG;
  }
#undef NSNKV_SEAL
  if (!done)
    seal_update_kernel<<<static_cast<unsigned>((batch + 255) / 256), 256, 0, st>>>(batch, tail_len, n_blocks, pending,
                                                                                   ts, tsh);
  return cudaGetLastError() == cudaSuccess ? NSNKV_OK : NSNKV_ERR_LAUNCH;
}

}  // namespace nsnkv

using namespace nsnkv;

extern "C" {

int nsnkv_version(void) { return 1; }

int64_t nsnkv_block_code_bytes(int bits) { return (bits >= 3 && bits <= 5) ? code_bytes(bits) : 0; }

int nsnkv_encode_blocks_strided(const void *x, int x_dtype, int64_t rows, int64_t blocks_per_row, int bits,
                                int norm_order, uint8_t *codes, uint8_t *q_out, uint16_t *norm, uint16_t *mn,
                                uint16_t *scale, uint8_t *headers, int64_t header_start, int64_t out_row_stride,
                                int64_t out_offset, int64_t blk_bytes, int code_order, int32_t *status, void *stream) {
  if (rows < 0 || blocks_per_row < 0 || bits < 3 || bits > 5 || (norm_order != 0 && norm_order != 1))
    return NSNKV_ERR_ARG;
  if (code_order < 0 || code_order > 2) return NSNKV_ERR_ARG;
  if (blk_bytes != 0 && (blk_bytes < code_bytes(bits) || blk_bytes % 16 != 0)) return NSNKV_ERR_ARG;
  const int64_t cs = blk_bytes ? blk_bytes : code_bytes(bits), ms = blk_bytes ? blk_bytes : kDim * 2;
  const int64_t n_blocks = rows * blocks_per_row;
  if (n_blocks == 0) return NSNKV_OK;
  if (n_blocks > 0x7FFFFFFF || !x || !norm || !mn || !scale || !status || !aligned16(x)) return NSNKV_ERR_ARG;
  if ((codes && !aligned16(codes)) || (q_out && !aligned16(q_out))) return NSNKV_ERR_ARG;
  if (out_offset < 0 || (rows > 1 && out_row_stride < blocks_per_row)) return NSNKV_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (x_dtype) {
    case NSNKV_F16:
      return launch_encode<__half>(x, n_blocks, blocks_per_row, bits, norm_order, codes, q_out, norm, mn, scale,
                                   headers, header_start, out_row_stride, out_offset, cs, ms, code_order, status, st);
    case NSNKV_BF16:
      return launch_encode<__nv_bfloat16>(x, n_blocks, blocks_per_row, bits, norm_order, codes, q_out, norm, mn,
                                          scale, headers, header_start, out_row_stride, out_offset, cs, ms, code_order, status, st);
    case NSNKV_F32:
      return launch_encode<float>(x, n_blocks, blocks_per_row, bits, norm_order, codes, q_out, norm, mn, scale,
                                  headers, header_start, out_row_stride, out_offset, cs, ms, code_order, status, st);
    default:
      return NSNKV_ERR_ARG;
  }
}

int nsnkv_encode_blocks(const void *x, int x_dtype, int64_t rows, int64_t blocks_per_row, int bits, int norm_order,
                        uint8_t *codes, uint8_t *q_out, uint16_t *norm, uint16_t *mn, uint16_t *scale,
                        uint8_t *headers, int64_t header_start, int64_t out_row_stride, int64_t out_offset,
                        int32_t *status, void *stream) {
  return nsnkv_encode_blocks_strided(x, x_dtype, rows, blocks_per_row, bits, norm_order, codes, q_out, norm, mn, scale,
                                     headers, header_start, out_row_stride, out_offset, 0, 0, status, stream);
}

int nsnkv_restore(const uint8_t *codes, int codes_unpacked, const uint16_t *norm, const uint16_t *mn,
                  const uint16_t *scale, int64_t rows, int64_t blocks_per_row, int bits, const void *tail,
                  int64_t tail_len, int dtype, void *out, int32_t *status, void *stream) {
  if (rows < 0 || blocks_per_row < 0 || tail_len < 0 || bits < 3 || bits > 5 || !out || !status) return NSNKV_ERR_ARG;
  if (rows * blocks_per_row > 0x7FFFFFFF) return NSNKV_ERR_ARG;
  if (rows * blocks_per_row > 0 && (!codes || !norm || !mn || !scale || !aligned16(codes))) return NSNKV_ERR_ARG;
  if (tail_len > 0 && !tail) return NSNKV_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case NSNKV_F16:
      return launch_restore<__half>(codes, codes_unpacked, norm, mn, scale, rows, blocks_per_row, bits, tail,
                                    tail_len, out, status, st);
    case NSNKV_BF16:
      return launch_restore<__nv_bfloat16>(codes, codes_unpacked, norm, mn, scale, rows, blocks_per_row, bits,
                                           tail, tail_len, out, status, st);
    case NSNKV_F32:
      return launch_restore<float>(codes, codes_unpacked, norm, mn, scale, rows, blocks_per_row, bits, tail,
                                   tail_len, out, status, st);
    default:
      return NSNKV_ERR_ARG;
  }
}

int nsnkv_pack(const uint8_t *codes, int64_t count, int bits, uint8_t *out, int32_t *status, void *stream) {
  if (count < 0 || bits < 3 || bits > 5) return NSNKV_ERR_ARG;
  if (count == 0) return NSNKV_OK;
  if (!codes || !out || !status) return NSNKV_ERR_ARG;
  int64_t groups = (count + 7) / 8;
  unsigned blocks = static_cast<unsigned>(std::min<int64_t>((groups + 255) / 256, 8192));
  pack_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(codes, count, bits, out, status);
  return cudaGetLastError() == cudaSuccess ? NSNKV_OK : NSNKV_ERR_LAUNCH;
}

int nsnkv_unpack(const uint8_t *payload, int64_t count, int bits, uint8_t *out, void *stream) {
  if (count < 0 || bits < 3 || bits > 5) return NSNKV_ERR_ARG;
  if (count == 0) return NSNKV_OK;
  if (!payload || !out) return NSNKV_ERR_ARG;
  int64_t groups = (count + 7) / 8;
  unsigned blocks = static_cast<unsigned>(std::min<int64_t>((groups + 255) / 256, 8192));
  unpack_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(payload, count, bits, out);
  return cudaGetLastError() == cudaSuccess ? NSNKV_OK : NSNKV_ERR_LAUNCH;
}

static int seal_impl(int64_t batch, int h, int bits, int dtype, void *k_tail, void *v_tail, int64_t tail_stride_seq,
                     int64_t tail_stride_head, int32_t *tail_len, int32_t *n_blocks, int pending_append,
                     const int32_t *block_table, int64_t table_stride, uint8_t *k_codes, uint16_t *k_norm,
                     uint16_t *k_min, uint16_t *k_scale, uint8_t *v_codes, uint16_t *v_norm, uint16_t *v_min,
                     uint16_t *v_scale, float *k_alpha, float *v_alpha, int64_t blk_bytes, int rec_order, int32_t *done,
                     int64_t blk_stride_head, int64_t blk_stride_page, int32_t *status, void *stream) {
  if (rec_order != 0 && rec_order != 1) return NSNKV_ERR_ARG;
  if (batch < 0 || h <= 0 || bits < 3 || bits > 5 || (pending_append != 0 && pending_append != 1)) return NSNKV_ERR_ARG;
  if (blk_bytes != 0 && (blk_bytes < code_bytes(bits) || blk_bytes % 16 != 0)) return NSNKV_ERR_ARG;
  const int64_t cs = blk_bytes ? blk_bytes : code_bytes(bits), ms = blk_bytes ? blk_bytes : kDim * 2;
  if (batch == 0) return NSNKV_OK;
  if (!k_tail || !v_tail || !tail_len || !n_blocks || !block_table || table_stride <= 0 || !k_codes || !v_codes ||
      !status)
    return NSNKV_ERR_ARG;
  if (!aligned16(k_tail) || !aligned16(v_tail) || !aligned16(k_codes) || !aligned16(v_codes)) return NSNKV_ERR_ARG;
  if ((k_alpha == nullptr) != (v_alpha == nullptr)) return NSNKV_ERR_ARG;
  if (tail_stride_head < kBlock || tail_stride_seq < tail_stride_head * h) return NSNKV_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case NSNKV_F16:
      return launch_seal<__half>(batch, h, bits, k_tail, v_tail, tail_stride_seq, tail_stride_head, tail_len,
                                 n_blocks, pending_append, block_table, table_stride, k_codes, k_norm, k_min,
                                 k_scale, v_codes, v_norm, v_min, v_scale, k_alpha, v_alpha, done, blk_stride_head,
                                 blk_stride_page, cs, ms, rec_order, status, st);
    case NSNKV_BF16:
      return launch_seal<__nv_bfloat16>(batch, h, bits, k_tail, v_tail, tail_stride_seq, tail_stride_head,
                                        tail_len, n_blocks, pending_append, block_table, table_stride, k_codes,
                                        k_norm, k_min, k_scale, v_codes, v_norm, v_min, v_scale, k_alpha, v_alpha,
                                        done, blk_stride_head, blk_stride_page, cs, ms, rec_order, status, st);
    default:
      return NSNKV_ERR_ARG;
  }
}

int nsnkv_seal_full_tails(int64_t batch, int h, int bits, int dtype, void *k_tail, void *v_tail,
                          int64_t tail_stride_seq, int64_t tail_stride_head, int32_t *tail_len, int32_t *n_blocks,
                          int pending_append, const int32_t *block_table, int64_t table_stride, uint8_t *k_codes,
                          uint16_t *k_norm, uint16_t *k_min, uint16_t *k_scale, uint8_t *v_codes, uint16_t *v_norm,
                          uint16_t *v_min, uint16_t *v_scale, int64_t blk_stride_head, int64_t blk_stride_page,
                          int32_t *status, void *stream) {
  return seal_impl(batch, h, bits, dtype, k_tail, v_tail, tail_stride_seq, tail_stride_head, tail_len, n_blocks,
                   pending_append, block_table, table_stride, k_codes, k_norm, k_min, k_scale, v_codes, v_norm,
                   v_min, v_scale, nullptr, nullptr, 0, 0, nullptr, blk_stride_head, blk_stride_page, status, stream);
}

int nsnkv_seal_full_tails_alpha(int64_t batch, int h, int bits, int dtype, void *k_tail, void *v_tail,
                                int64_t tail_stride_seq, int64_t tail_stride_head, int32_t *tail_len,
                                int32_t *n_blocks, int pending_append, const int32_t *block_table,
                                int64_t table_stride, uint8_t *k_codes, uint16_t *k_norm, uint16_t *k_min,
                                uint16_t *k_scale, uint8_t *v_codes, uint16_t *v_norm, uint16_t *v_min,
                                uint16_t *v_scale, float *k_alpha, float *v_alpha, int64_t blk_bytes, int rec_order,
                                int32_t *seq_counters, int64_t blk_stride_head, int64_t blk_stride_page,
                                int32_t *status, void *stream) {
  if (!k_alpha || !v_alpha) return NSNKV_ERR_ARG;
  return seal_impl(batch, h, bits, dtype, k_tail, v_tail, tail_stride_seq, tail_stride_head, tail_len, n_blocks,
                   pending_append, block_table, table_stride, k_codes, k_norm, k_min, k_scale, v_codes, v_norm,
                   v_min, v_scale, k_alpha, v_alpha, blk_bytes, rec_order, seq_counters, blk_stride_head,
                   blk_stride_page, status, stream);
}

int nsnkv_block_renorm(int bits, int64_t rows, int64_t blocks_per_row, const uint8_t *codes, const uint16_t *norm,
                       const uint16_t *min, const uint16_t *scale, int64_t row_stride, int64_t offset, float *alpha,
                       int64_t blk_bytes, int code_order, void *stream) {
  if (bits < 3 || bits > 5 || rows < 0 || blocks_per_row < 0 || offset < 0) return NSNKV_ERR_ARG;
  if (code_order < 0 || code_order > 2) return NSNKV_ERR_ARG;
  if (blk_bytes != 0 && (blk_bytes < code_bytes(bits) || blk_bytes % 16 != 0)) return NSNKV_ERR_ARG;
  const int64_t cs = blk_bytes ? blk_bytes : code_bytes(bits), ms = blk_bytes ? blk_bytes : kDim * 2;
  if (rows == 0 || blocks_per_row == 0) return NSNKV_OK;
  if (!codes || !norm || !min || !scale || !alpha || row_stride < blocks_per_row + offset) return NSNKV_ERR_ARG;
  if (rows * blocks_per_row > 0x7fffffffLL) return NSNKV_ERR_TOO_LARGE;
  const unsigned grid = static_cast<unsigned>(rows * blocks_per_row);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (bits) {
    case 3:
      renorm_blocks_kernel<3><<<grid, 256, 0, st>>>(codes, norm, min, scale, blocks_per_row, row_stride, offset,
                                                     alpha, cs, ms, code_order);
      break;
    case 4:
      renorm_blocks_kernel<4><<<grid, 256, 0, st>>>(codes, norm, min, scale, blocks_per_row, row_stride, offset,
                                                     alpha, cs, ms, code_order);
      break;
    default:
      renorm_blocks_kernel<5><<<grid, 256, 0, st>>>(codes, norm, min, scale, blocks_per_row, row_stride, offset,
                                                     alpha, cs, ms, code_order);
      break;
  }
  return cudaGetLastError() == cudaSuccess ? NSNKV_OK : NSNKV_ERR_LAUNCH;
}

}  // extern "C"
