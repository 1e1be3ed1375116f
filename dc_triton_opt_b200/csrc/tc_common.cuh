// Shared pieces of the tensor-core DC-attention kernels (sm_100a):
// tile constants, kernel parameters, the cross-head composition of one
// (query, key) pair, per-key weight loads, and the host-side TMA tensor maps.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <type_traits>

#include "common.cuh"
#include "sm100_ptx.cuh"

namespace dcattn {
namespace tc {


constexpr int NQ = 128;          // (head, query) columns per CTA
constexpr int KT_ROWS = 128;     // keys per key tile (TMEM lanes)
constexpr int TILE_BYTES = KT_ROWS * 128 * 2;  // one K or V tile: 128 rows x 128 d x 2 B
constexpr int D = 128;

enum Err { ERR_TIMEOUT_Q = 1, ERR_TIMEOUT_FULL = 2, ERR_TIMEOUT_FREE = 3, ERR_TIMEOUT_S = 4,
           ERR_TIMEOUT_P = 5, ERR_TIMEOUT_O = 6 };

struct Geo {
  int nkt, nslot;
  int q_off, ring_off, p_off, misc_off;
  int rec_off, mrec_off, red_off, fac_off, bar_off, tmem_off;
  int total;
};

__host__ __device__ constexpr int round_up(int x, int a) { return (x + a - 1) / a * a; }

// Shared memory of the one-tile-per-CTA kernel (dc_tc_kernel).
__host__ __device__ inline Geo make_geo(int HPG, int R, int nkt) {
  Geo g{};
  const int BM = NQ / HPG;
  g.nkt = nkt;
  g.nslot = nkt == 3 ? 2 : 3;
  g.q_off = 0;
  g.ring_off = g.q_off + NQ * 256;
  g.p_off = g.ring_off + g.nslot * TILE_BYTES;
  g.misc_off = g.p_off + nkt * NQ * KT_ROWS * 2;
  int o = g.misc_off;
  g.rec_off = round_up(o, 16); o = g.rec_off + 2 * BM * HPG * (2 * R + 1) * 4;  // per-query weights
  g.mrec_off = round_up(o, 16); o = g.mrec_off + 2 * BM * HPG * HPG * 4;         // mixing matrices
  g.red_off = round_up(o, 16); o = g.red_off + 2 * 4 * nkt * NQ * 4;             // column maxima | sums
  g.fac_off = o; o += 4 * nkt * NQ * 4;                                          // probability factors
  g.bar_off = round_up(o, 8); o = g.bar_off + 16 * 8;
  g.tmem_off = o; o += 16;
  g.total = o;
  return g;
}

struct TermPtrs {
  int identity;
  const float *w;
  const void *qw1, *qw2, *kw1, *kw2, *qdd, *kdd;
  const void *qmat;  // [B, T, H, HPG] per-query mix inside the group (decomposed form)
};

struct TcParams {
  int B, T, H, G, window, slen_default;
  float scale;
  const int32_t *seq_lens;
  void *out;
  int64_t out_sb, out_st, out_sh;
  int32_t *err_flag;
  uint32_t wait_us;  // limit of every mbarrier wait (microseconds)
  int32_t skip_loads;  // testing: the TMA producer issues nothing (waits run out)
  TermPtrs pre, post;
};

// A bounded wait that ran out writes its code here (the first code wins).
// err_flag is never NULL in a launch: the C layer substitutes the library's
// per-device error word when the caller passes none.
__device__ __forceinline__ void record_err(const TcParams &p, int code) {
  atomicCAS(p.err_flag, 0, code);
}

// Static head mix of a group, stored transposed with a zero diagonal:
// wt[h * HPG + hp] = w[g, hp, h] for hp != h.  Up to HPG = 4 it is held in
// registers; for larger groups it is read from shared memory (broadcast float4
// loads) to keep the compose threads free of register spills.
template <int HPG, bool REG = (HPG <= 4)>
struct WSrc;
template <int HPG>
struct WSrc<HPG, true> {
  float v[HPG * HPG];
  __device__ __forceinline__ void load(const float *smem_wt) {
#pragma unroll
    for (int j = 0; j < HPG * HPG; ++j) v[j] = smem_wt[j];
  }
  __device__ __forceinline__ void row(int h, float (&r)[HPG]) const {
#pragma unroll
    for (int hp = 0; hp < HPG; ++hp) r[hp] = v[h * HPG + hp];
  }
};
template <int HPG>
struct WSrc<HPG, false> {
  const float *p;
  __device__ __forceinline__ void load(const float *smem_wt) { p = smem_wt; }
  __device__ __forceinline__ void row(int h, float (&r)[HPG]) const {
#pragma unroll
    for (int hp = 0; hp < HPG; hp += 4) {
      const float4 x = *reinterpret_cast<const float4 *>(p + h * HPG + hp);
      r[hp] = x.x; r[hp + 1] = x.y; r[hp + 2] = x.z; r[hp + 3] = x.w;
    }
  }
};

// Composition of one (query, key) pair across the HPG heads of a group.
// a: per-head inputs; W: static mix (transposed, zero diagonal); rec:
// per-query record (dq = w[h,h] + identity + qdd[t,h]; qa = qw1[t,:,r];
// qb = qw2[t,r,:]); kw1/kw2/kdd: per-key weights of this thread's key.
template <int HPG, int R>
__device__ __forceinline__ void compose(const float (&a)[HPG], float (&o)[HPG], const WSrc<HPG> &W,
                                        const float *rec, const float (&kw1)[HPG * R],
                                        const float (&kw2)[R * HPG], const float (&kdd)[HPG]) {
  float r4[round_up(HPG * (2 * R + 1), 4)];
#pragma unroll
  for (int j = 0; j < round_up(HPG * (2 * R + 1), 4); j += 4) {
    const float4 x = *reinterpret_cast<const float4 *>(rec + j);
    r4[j] = x.x; r4[j + 1] = x.y; r4[j + 2] = x.z; r4[j + 3] = x.w;
  }
  const float *dq = r4, *qa = r4 + HPG, *qb = r4 + HPG + HPG * R;
  float aq[R], ak[R];
#pragma unroll
  for (int r = 0; r < R; ++r) { aq[r] = 0.f; ak[r] = 0.f; }
#pragma unroll
  for (int h = 0; h < HPG; ++h) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      aq[r] = fmaf(qa[h * R + r], a[h], aq[r]);
      ak[r] = fmaf(kw1[h * R + r], a[h], ak[r]);
    }
  }
#pragma unroll
  for (int h = 0; h < HPG; ++h) {
    float wr[HPG];
    W.row(h, wr);
    float x = (dq[h] + kdd[h]) * a[h];
#pragma unroll
    for (int hp = 0; hp < HPG; ++hp)
      if (hp != h) x = fmaf(wr[hp], a[hp], x);
#pragma unroll
    for (int r = 0; r < R; ++r) x = fmaf(qb[r * HPG + h], aq[r], fmaf(kw2[r * HPG + h], ak[r], x));
    o[h] = x;
  }
}

// Paired form of compose for two queries (pair half x: query i, y: query
// i + 1) against the thread's key, on .f32x2 instructions.  Every half
// performs the same operations in the same order as compose, so the results
// are bit-identical.  rec2 is the pair-interleaved record of the two queries:
// rec2[2 j + q] = element j of query q's record.  The per-key weights and the
// static mix are held as duplicated pairs.  The pairs need about twice the
// registers of the scalar form: at 2 or more heads per group the persistent
// kernel then spills and runs slower, so only the 1-head groups use it.
template <int HPG, int R>
struct KeyW2 {
  ptx::f2_t kw1[HPG * R], kw2[R * HPG], kdd[HPG];
  __device__ __forceinline__ void set(const float (&a)[HPG * R], const float (&b)[R * HPG], const float (&c)[HPG]) {
#pragma unroll
    for (int j = 0; j < HPG * R; ++j) { kw1[j] = ptx::f2_dup(a[j]); kw2[j] = ptx::f2_dup(b[j]); }
#pragma unroll
    for (int j = 0; j < HPG; ++j) kdd[j] = ptx::f2_dup(c[j]);
  }
};
template <int HPG>
struct WSrc2 {
  const float *p;
  __device__ __forceinline__ void load(const float *smem_wt) { p = smem_wt; }
  __device__ __forceinline__ ptx::f2_t get(int h, int hp) const { return ptx::f2_dup(p[h * HPG + hp]); }
};

template <int HPG, int R>
__device__ __forceinline__ void compose2(const ptx::f2_t (&a)[HPG], ptx::f2_t (&o)[HPG], const WSrc2<HPG> &W,
                                         const float *rec2, const KeyW2<HPG, R> &K) {
  constexpr int RF = round_up(HPG * (2 * R + 1), 4);
  ptx::f2_t r2[RF];
#pragma unroll
  for (int j = 0; j < RF; j += 2) {
    const float4 x = *reinterpret_cast<const float4 *>(rec2 + 2 * j);
    r2[j] = ptx::f2_pack(x.x, x.y);
    r2[j + 1] = ptx::f2_pack(x.z, x.w);
  }
  const ptx::f2_t *dq = r2, *qa = r2 + HPG, *qb = r2 + HPG + HPG * R;
  ptx::f2_t aq[R], ak[R];
#pragma unroll
  for (int r = 0; r < R; ++r) { aq[r] = 0ull; ak[r] = 0ull; }
#pragma unroll
  for (int h = 0; h < HPG; ++h) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      aq[r] = ptx::f2_fma(qa[h * R + r], a[h], aq[r]);
      ak[r] = ptx::f2_fma(K.kw1[h * R + r], a[h], ak[r]);
    }
  }
#pragma unroll
  for (int h = 0; h < HPG; ++h) {
    ptx::f2_t x = ptx::f2_mul(ptx::f2_add(dq[h], K.kdd[h]), a[h]);
#pragma unroll
    for (int hp = 0; hp < HPG; ++hp)
      if (hp != h) x = ptx::f2_fma(W.get(h, hp), a[hp], x);
#pragma unroll
    for (int r = 0; r < R; ++r) x = ptx::f2_fma(qb[r * HPG + h], aq[r], ptx::f2_fma(K.kw2[r * HPG + h], ak[r], x));
    o[h] = x;
  }
}

// Logit given to masked (query, key) pairs: finite, so that max / exp need no
// infinity checks; 2^(kMaskedLogit - m) is 0 for any real maximum m.
constexpr float kMaskedLogit = -1e30f;

// HPG consecutive floats of shared memory (16-byte aligned when HPG % 4 == 0).
template <int HPG>
__device__ __forceinline__ void ld_row(const float *p, float (&r)[HPG]) {
  if constexpr (HPG % 4 == 0) {
#pragma unroll
    for (int j = 0; j < HPG; j += 4) {
      const float4 x = *reinterpret_cast<const float4 *>(p + j);
      r[j] = x.x; r[j + 1] = x.y; r[j + 2] = x.z; r[j + 3] = x.w;
    }
  } else if constexpr (HPG == 2) {
    const float2 x = *reinterpret_cast<const float2 *>(p);
    r[0] = x.x; r[1] = x.y;
  } else {
    r[0] = p[0];
  }
}

// Composition of one (query, key) pair with the query's mixing matrix M
// (shared memory, [h'][h]: the coefficient of a[h'] in o[h]) and the key's
// weights in registers:
//   o[h] = sum_h' M[h'][h] a[h'] + kdd[h] a[h] + sum_r kw2[r][h] sum_h' kw1[h'][r] a[h'].
template <int HPG, int R>
__device__ __forceinline__ void compose_m(const float (&a)[HPG], float (&o)[HPG], const float *M,
                                          const float (&kw1)[HPG * R], const float (&kw2)[R * HPG],
                                          const float (&kdd)[HPG]) {
  float ak[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    ak[r] = 0.f;
#pragma unroll
    for (int h = 0; h < HPG; ++h) ak[r] = fmaf(kw1[h * R + r], a[h], ak[r]);
  }
#pragma unroll
  for (int h = 0; h < HPG; ++h) o[h] = kdd[h] * a[h];
#pragma unroll
  for (int h1 = 0; h1 < HPG; ++h1) {
    float mr[HPG];
    ld_row<HPG>(M + h1 * HPG, mr);
#pragma unroll
    for (int h = 0; h < HPG; ++h) o[h] = fmaf(mr[h], a[h1], o[h]);
  }
#pragma unroll
  for (int h = 0; h < HPG; ++h)
#pragma unroll
    for (int r = 0; r < R; ++r) o[h] = fmaf(kw2[r * HPG + h], ak[r], o[h]);
}

// compose_m for two queries at once on paired fp32 (.f32x2): lane x of a pair
// is query i, lane y query i + 1; M2 holds the two queries' matrices
// interleaved, [h'][h][query].  Per-key weights are duplicated pairs.  Each
// half performs the operations of compose_m in the same order.
template <int HPG, int R>
__device__ __forceinline__ void compose_m2(const ptx::f2_t (&a)[HPG], ptx::f2_t (&o)[HPG], const float *M2,
                                           const ptx::f2_t (&kw1)[HPG * R], const ptx::f2_t (&kw2)[R * HPG],
                                           const ptx::f2_t (&kdd)[HPG]) {
  ptx::f2_t ak[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    ak[r] = 0ull;
#pragma unroll
    for (int h = 0; h < HPG; ++h) ak[r] = ptx::f2_fma(kw1[h * R + r], a[h], ak[r]);
  }
#pragma unroll
  for (int h = 0; h < HPG; ++h) o[h] = ptx::f2_mul(kdd[h], a[h]);
#pragma unroll
  for (int h1 = 0; h1 < HPG; ++h1) {
    float mr[2 * HPG];
    ld_row<2 * HPG>(M2 + h1 * 2 * HPG, mr);
#pragma unroll
    for (int h = 0; h < HPG; ++h) o[h] = ptx::f2_fma(ptx::f2_pack(mr[2 * h], mr[2 * h + 1]), a[h1], o[h]);
  }
#pragma unroll
  for (int h = 0; h < HPG; ++h)
#pragma unroll
    for (int r = 0; r < R; ++r) o[h] = ptx::f2_fma(kw2[r * HPG + h], ak[r], o[h]);
}

// Two floats rounded to E (bf16 / fp16) and packed low | high << 16.
template <typename E>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const E a = from_f<E>(lo), b = from_f<E>(hi);
  return static_cast<uint32_t>(*reinterpret_cast<const uint16_t *>(&a)) |
         (static_cast<uint32_t>(*reinterpret_cast<const uint16_t *>(&b)) << 16);
}

template <typename E>
__device__ __forceinline__ float ld_w(const void *base, int64_t idx) {
  return to_f<E>(reinterpret_cast<const E *>(base)[idx]);
}

// Entry (h1 -> h) of query t's per-query mix: the weight of a[h1] in the
// composed value of head h, qmat[b, t, hbase + h, h1] (dc_attention_torch.py:59-61
// mixes logits as mixed[i] = sum_j pre_w[i, j] L[j]); 0 without qmat or for
// t outside the sequence.
template <typename E>
__device__ __forceinline__ float qmat_at(const TermPtrs &tm, int b, int t, int T, int H, int hpg, int hbase, int h1,
                                         int h) {
  if (!tm.qmat || t >= T) return 0.f;
  return ld_w<E>(tm.qmat, (((int64_t)b * T + t) * H + hbase + h) * hpg + h1);
}

// N consecutive 16-bit elements (N * 2 bytes, aligned to that size), raw.
template <int N>
struct Raw16 {
  uint32_t w[(N + 1) / 2];
};
template <int N>
__device__ __forceinline__ Raw16<N> ld_raw16(const void *p) {
  Raw16<N> r;
  if constexpr (N == 1) {
    r.w[0] = __ldg(reinterpret_cast<const unsigned short *>(p));
  } else if constexpr (N == 2) {
    r.w[0] = __ldg(reinterpret_cast<const unsigned int *>(p));
  } else if constexpr (N == 4) {
    const uint2 x = __ldg(reinterpret_cast<const uint2 *>(p));
    r.w[0] = x.x; r.w[1] = x.y;
  } else {
    static_assert(N % 8 == 0, "16-bit vector of 1, 2, 4 or a multiple of 8 elements");
#pragma unroll
    for (int k = 0; k < N / 8; ++k) {
      const uint4 x = __ldg(reinterpret_cast<const uint4 *>(p) + k);
      r.w[4 * k] = x.x; r.w[4 * k + 1] = x.y; r.w[4 * k + 2] = x.z; r.w[4 * k + 3] = x.w;
    }
  }
  return r;
}
template <int N>
__device__ __forceinline__ Raw16<N> raw16_zero() {
  Raw16<N> r;
#pragma unroll
  for (int k = 0; k < (N + 1) / 2; ++k) r.w[k] = 0u;
  return r;
}
// element i of a raw vector as float (the bit pattern 0 converts to 0.0)
template <typename E, int N>
__device__ __forceinline__ float raw16_get(const Raw16<N> &r, int i) {
  const unsigned short b = static_cast<unsigned short>(r.w[i >> 1] >> (16 * (i & 1)));
  return to_f<E>(*reinterpret_cast<const E *>(&b));
}
template <typename E>
__device__ __forceinline__ const E *elem(const void *base, int64_t i) {
  return reinterpret_cast<const E *>(base) + i;
}

// The per-key weights of key token `tok` for heads [hbase, hbase + HPG): kw1
// [h][r], kw2 [r][h], kdd [h], each a run of contiguous elements loaded as one
// vector (zero when the key is outside the sequence or the term is absent).
template <typename E, int HPG, int R>
__device__ __forceinline__ void load_key_weights_vec(const TermPtrs &tm, int64_t tok, int H, int hbase, bool ok,
                                                     float (&kw1)[HPG * R], float (&kw2)[R * HPG],
                                                     float (&kdd)[HPG]) {
  const Raw16<HPG * R> a = (ok && tm.kw1) ? ld_raw16<HPG * R>(elem<E>(tm.kw1, (tok * H + hbase) * R))
                                          : raw16_zero<HPG * R>();
  const Raw16<HPG> c = (ok && tm.kdd) ? ld_raw16<HPG>(elem<E>(tm.kdd, tok * H + hbase)) : raw16_zero<HPG>();
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const Raw16<HPG> bq = (ok && tm.kw2) ? ld_raw16<HPG>(elem<E>(tm.kw2, (tok * R + r) * H + hbase))
                                         : raw16_zero<HPG>();
#pragma unroll
    for (int h = 0; h < HPG; ++h) kw2[r * HPG + h] = raw16_get<E, HPG>(bq, h);
  }
#pragma unroll
  for (int j = 0; j < HPG * R; ++j) kw1[j] = raw16_get<E, HPG * R>(a, j);
#pragma unroll
  for (int h = 0; h < HPG; ++h) kdd[h] = raw16_get<E, HPG>(c, h);
}

template <typename E, int HPG, int R>
__device__ __forceinline__ void load_key_weights(const TermPtrs &tm, int64_t tok, int H, int hbase, bool ok,
                                                 float (&kw1)[HPG * R], float (&kw2)[R * HPG],
                                                 float (&kdd)[HPG]) {
#pragma unroll
  for (int h = 0; h < HPG; ++h) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      kw1[h * R + r] = (ok && tm.kw1) ? ld_w<E>(tm.kw1, (tok * H + hbase + h) * R + r) : 0.f;
      kw2[r * HPG + h] = (ok && tm.kw2) ? ld_w<E>(tm.kw2, (tok * R + r) * H + hbase + h) : 0.f;
    }
    kdd[h] = (ok && tm.kdd) ? ld_w<E>(tm.kdd, tok * H + hbase + h) : 0.f;
  }
}


typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// [B, T, H, D] tensor (element strides sb, st, sh; d contiguous) as a 4-D map
// (D, H, T, B); box = 64 d x 1 head x rows x 1.
static bool make_map(CUtensorMap *m, const void *base, int dtype, int B, int T, int H, int rows, int64_t sb,
                     int64_t st, int64_t sh, bool swizzle) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)sh * 2, (cuuint64_t)st * 2, (cuuint64_t)sb * 2};
  const cuuint32_t box[4] = {64, 1, (cuuint32_t)rows, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt =
      dtype == DC_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return enc(m, dt, 4, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A [B, T, H, D] tensor of 8-bit floats (e4m3) as a 4-D map whose box is one
// head's full 128-byte rows (128 d x rows), 128-byte swizzled.
static bool make_map8(CUtensorMap *m, const void *base, int B, int T, int H, int rows, int64_t sb, int64_t st,
                      int64_t sh) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)sh, (cuuint64_t)st, (cuuint64_t)sb};
  const cuuint32_t box[4] = {128, 1, (cuuint32_t)rows, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void *>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The same [B, T, H, D] tensor as a 5-D map (64 d, T, d half, H, B) whose box
// (64 x rows x 2 x heads x 1) lands in shared memory as [head][d half][rows][64 d]:
// one TMA operation fills both 128-byte-swizzled d halves of `heads` heads.
// (One thread's TMA operations are processed one after another; fewer, larger
// boxes and several issuing lanes are what raise the per-SM load rate.)
static bool make_map5(CUtensorMap *m, const void *base, int dtype, int B, int T, int H, int rows, int heads,
                      int64_t sb, int64_t st, int64_t sh) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return false;
  const cuuint64_t dims[5] = {64, (cuuint64_t)T, 2, (cuuint64_t)H, (cuuint64_t)B};
  const cuuint64_t strides[4] = {(cuuint64_t)st * 2, 128, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
  const cuuint32_t box[5] = {64, (cuuint32_t)rows, 2, (cuuint32_t)heads, 1};
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUtensorMapDataType dt =
      dtype == DC_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return enc(m, dt, 5, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// key span of a query block: BM + window - 1 keys
static int num_key_tiles(int HPG, int window) {
  const int BM = NQ / HPG;
  return (BM + window - 1 + KT_ROWS - 1) / KT_ROWS;
}
// rows of the last key tile, rounded up to the 16-key MMA step
static int last_tile_rows(int HPG, int window) {
  const int BM = NQ / HPG;
  const int span = BM + window - 1;
  const int r = span - KT_ROWS * (num_key_tiles(HPG, window) - 1);
  return (r + 15) / 16 * 16;
}

static TermPtrs to_ptrs(const dc_terms &t) {
  TermPtrs r;
  r.identity = t.identity;
  r.w = t.w;
  r.qw1 = t.qw1; r.qw2 = t.qw2; r.kw1 = t.kw1; r.kw2 = t.kw2; r.qdd = t.qdd; r.kdd = t.kdd;
  r.qmat = t.qmat;
  return r;
}


static int sm_count() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!n[dev]) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  return n[dev] > 0 ? n[dev] : 148;
}

}  // namespace tc
}  // namespace dcattn
