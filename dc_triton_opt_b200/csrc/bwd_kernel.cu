// Backward of the DC-attention forward (sm_100a, CUDA cores, fp32).
//
// Reference: TritonDCResidual.backward (triton_dc_residual.py:1707-1892), the
// residual rank-1 form with six [B,T,N] weights; this kernel covers the
// query-side term family of the forward: identity, static mix w, rank-R
// query-wise qw1/qw2, qdd gates and per-query matrices qmat, pre and post,
// windowed layers (and full-causal ones short enough for one block).
//
// For a query t and the HPG heads of its group every query-side term folds
// into one matrix per set, M_t[h'][h] (weight of a[h'] in the composed value
// of head h).  Forward, per key s of t's window:
//   L[h]  = scale q_h(t).k_h(s)
//   S[h]  = sum_h' Mpre_t[h'][h] L[h']             (masked after composition)
//   P     = softmax_s(S)                            (fully masked row -> 0)
//   P'[h] = sum_h' Mpost_t[h'][h] P[h']
//   O_h   = sum_s P'[h] v_h(s)
// Backward (dO given):
//   dV_h(s) += P'[h] dO_h           dP'[h] = dO_h.v_h(s)
//   dP[h']   = sum_h Mpost[h'][h] dP'[h]        dMpost[h'][h] = sum_s P[h'] dP'[h]
//   dS[h]    = P[h] (dP[h] - sum_s P[h] dP[h])
//   dL[h']   = sum_h Mpre[h'][h] dS[h]          dMpre[h'][h]  = sum_s L[h'] dS[h]
//   dQ_h     = scale sum_s dL[h] k_h(s)         dK_h(s) += scale dL[h] q_h
// and the weight gradients follow from dM: dqdd[h] = dM[h][h],
// dqw1[h'][r] = sum_h dM[h'][h] qw2[r][h], dqw2[r][h] = sum_h' qw1[h'][r] dM[h'][h],
// dqmat[h][h'] = dM[h'][h], dw[g] = sum over (b, t) of dM.
//
// One CTA owns (batch b, head group g, BM queries) and every key of their
// windows, so the softmax statistics, the row sums and all per-query
// gradients are block-local (nothing saved by the forward is needed).  Keys
// are shared with neighbouring blocks: dK and dV are accumulated in fp32 by
// vector atomic adds (one per 4 elements after the block's own reduction),
// as the reference also returns them in fp32.  L, P (then dS) and P' (then
// dP', dP) live in shared memory as [column = (head, query)][key] planes; one
// head's K or V rows of the key span are staged at a time.

#include <cuda_runtime.h>

#include <string>
#include <type_traits>

#include "common.cuh"

namespace dcattn {
namespace bwd {

constexpr int D = 128;
constexpr int DP = D + 8;     // padded smem row of a q / dO / k / v row (elements): 16-byte loads conflict-free
constexpr int NT = 512;       // threads per CTA
constexpr int MAX_SMEM = 227 * 1024;

struct Geo {
  int BM, NC, span, SP, SPR;
  int l_off, p_off, d_off, q_off, do_off, kv_off, m_off, rec_off, total;
};

__host__ __device__ inline int rup(int x, int a) { return (x + a - 1) / a * a; }

template <int HPG, int R>
__host__ __device__ inline Geo make_geo(int BM, int W, int esize) {
  Geo g{};
  g.BM = BM;
  g.NC = BM * HPG;
  g.span = BM + W - 1;
  g.SPR = rup(g.span, 32);
  // row length = 4 mod 32: the tensor-core fragment accesses (lanes g = 0..7
  // along keys, t = 0..3 along rows two apart) fall on 32 distinct banks
  g.SP = g.SPR + 4;
  int o = 0;
  g.l_off = o; o += g.NC * g.SP * 4;                     // L, then dL
  g.p_off = o; o += g.NC * g.SP * 4;                     // S, then P
  g.d_off = o; o += g.NC * g.SP * 4;                     // P', dP', dP, then dS
  o = rup(o, 16);
  // row counts padded so that 16-row tensor-core fragments never leave a region
  // (the pad rows are zeroed once and never written)
  g.q_off = o; o += (rup(g.NC, 16) + 16) * DP * esize;   // q rows
  g.do_off = o; o += (rup(g.NC, 16) + 16) * DP * esize;  // dO rows
  // one head's K or V rows of the span; dM (the mixing-matrix gradient of one
  // set) shares this region: it is live only between the head loops, while
  // no K or V rows are staged
  const int kv_bytes = (rup(g.span, 16) + 16) * DP * esize, dm_bytes = BM * HPG * HPG * 4;
  g.kv_off = o; o += kv_bytes > dm_bytes ? kv_bytes : dm_bytes;
  o = rup(o, 16);
  g.m_off = o; o += 2 * BM * HPG * HPG * 4;              // Mpre, Mpost
  g.rec_off = o; o += 2 * 2 * BM * HPG * R * 4;          // [set][qw1 | qw2][BM][HPG * R]
  g.total = o;
  return g;
}

__device__ __forceinline__ void red_add_v4(float *addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// ---- warp-level tensor-core products (mma.sync m16n8k16, fp32 accumulate).
// Fragment layout (g = lane / 4, t = lane % 4): A 16x16 row-major as
// a0 (g, 2t..2t+1), a1 (g+8, 2t..), a2 (g, 2t+8..), a3 (g+8, 2t+8..);
// B 16x8 as b0 (k 2t..2t+1, n g), b1 (k 2t+8.., n g); C 16x8 as
// c0 c1 (g, 2t..2t+1), c2 c3 (g+8, 2t..2t+1).
template <typename E>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  if constexpr (std::is_same<E, __nv_bfloat16>::value)
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  else
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t (&r)[2], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1]) : "r"(smem_u32(p)));
}

template <typename E>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  E a = from_f<E>(lo), b = from_f<E>(hi);
  return static_cast<uint32_t>(*reinterpret_cast<uint16_t *>(&a)) |
         (static_cast<uint32_t>(*reinterpret_cast<uint16_t *>(&b)) << 16);
}

__device__ __forceinline__ void red_add_v2(float *addr, float a, float b) {
  asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(addr), "f"(a), "f"(b) : "memory");
}

template <typename E>
__device__ __forceinline__ void ld8(const E *p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4 *>(p);
  const E *e = reinterpret_cast<const E *>(&u);
#pragma unroll
  for (int k = 0; k < 8; ++k) f[k] = to_f<E>(e[k]);
}

struct TermG {
  float *w, *qw1, *qw2, *qdd, *qmat;
};

struct BwdParams {
  int B, T, H, G, R, window;  // window: effective W (>= 1)
  float scale;
  const void *q, *k, *v, *dout;
  const int32_t *seq_lens;
  void *dq;
  float *dk, *dv;
  TermsDev pre, post;
  TermG gpre, gpost;
};

template <typename E, int HPG, int R>
__global__ void __launch_bounds__(NT, 1) dc_bwd_kernel(const BwdParams p, const Geo geo) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int BM = geo.BM, NC = geo.NC, span = geo.span, SP = geo.SP, SPR = geo.SPR;
  float *Lb = reinterpret_cast<float *>(smem + geo.l_off);
  float *Pb = reinterpret_cast<float *>(smem + geo.p_off);
  float *Db = reinterpret_cast<float *>(smem + geo.d_off);
  E *Qs = reinterpret_cast<E *>(smem + geo.q_off);
  E *dOs = reinterpret_cast<E *>(smem + geo.do_off);
  E *KVs = reinterpret_cast<E *>(smem + geo.kv_off);
  float *Mpre = reinterpret_cast<float *>(smem + geo.m_off);
  float *Mpost = Mpre + BM * HPG * HPG;
  float *dM = reinterpret_cast<float *>(smem + geo.kv_off);
  float *rec = reinterpret_cast<float *>(smem + geo.rec_off);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.y / p.G, g = blockIdx.y % p.G;
  const int T = p.T, H = p.H, W = p.window, hbase = g * HPG;
  const int q0 = blockIdx.x * BM, k_lo = q0 - W + 1;
  const int slen = p.seq_lens ? min(max(p.seq_lens[b], 0), T) : T;
  const E *qg = reinterpret_cast<const E *>(p.q), *kg = reinterpret_cast<const E *>(p.k);
  const E *vg = reinterpret_cast<const E *>(p.v), *dog = reinterpret_cast<const E *>(p.dout);
  auto row = [&](int t, int h) -> int64_t { return (((int64_t)b * T + t) * H + hbase + h) * D; };
  auto valid = [&](int t, int s) { return s >= 0 && s < slen && s <= t && t - s < W && t < T; };

  // ---- q and dO rows of the block, per-query weights, mixing matrices
  for (int idx = tid; idx < NC * (D / 8); idx += NT) {
    const int c = idx / (D / 8), ch = idx % (D / 8), h = c / BM, t = q0 + c % BM;
    uint4 uq = make_uint4(0, 0, 0, 0), ud = uq;
    if (t < T) {
      uq = *reinterpret_cast<const uint4 *>(qg + row(t, h) + ch * 8);
      ud = *reinterpret_cast<const uint4 *>(dog + row(t, h) + ch * 8);
    }
    *reinterpret_cast<uint4 *>(Qs + c * DP + ch * 8) = uq;
    *reinterpret_cast<uint4 *>(dOs + c * DP + ch * 8) = ud;
  }
  {
    const int nq = rup(NC, 16) + 16, nkv = rup(span, 16) + 16;
    for (int idx = tid; idx < (nq - NC) * (DP / 8); idx += NT) {
      const int r = NC + idx / (DP / 8), ch = idx % (DP / 8);
      *reinterpret_cast<uint4 *>(Qs + r * DP + ch * 8) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4 *>(dOs + r * DP + ch * 8) = make_uint4(0, 0, 0, 0);
    }
    for (int idx = tid; idx < (nkv - span) * (DP / 8); idx += NT) {
      const int r = span + idx / (DP / 8), ch = idx % (DP / 8);
      *reinterpret_cast<uint4 *>(KVs + r * DP + ch * 8) = make_uint4(0, 0, 0, 0);
    }
  }
  for (int idx = tid; idx < 2 * 2 * BM * HPG * R; idx += NT) {
    const int set = idx / (2 * BM * HPG * R), part = (idx / (BM * HPG * R)) % 2, rem = idx % (BM * HPG * R);
    const int i = rem / (HPG * R), t = q0 + i;
    const TermsDev &tm = set ? p.post : p.pre;
    float val = 0.f;
    if (t < T && tm.qw1) {
      const int64_t tok = (int64_t)b * T + t;
      if (part == 0) {  // qw1[t][h][r], flat (h, r)
        const int h = (rem % (HPG * R)) / R, r = rem % R;
        val = ldw<E>(tm.qw1, (tok * H + hbase + h) * R + r);
      } else {  // qw2[t][r][h], flat (r, h)
        const int r = (rem % (HPG * R)) / HPG, h = rem % HPG;
        val = ldw<E>(tm.qw2, (tok * R + r) * H + hbase + h);
      }
    }
    rec[idx] = val;
  }
  __syncthreads();
  for (int idx = tid; idx < 2 * BM * HPG * HPG; idx += NT) {
    const int set = idx / (BM * HPG * HPG), i = (idx / (HPG * HPG)) % BM, h1 = (idx / HPG) % HPG, h = idx % HPG;
    const TermsDev &tm = set ? p.post : p.pre;
    const int t = q0 + i;
    float m = 0.f;
    if (t < T) {
      const int64_t tok = (int64_t)b * T + t;
      m = (tm.w ? tm.w[((int64_t)g * HPG + h1) * HPG + h] : 0.f);
      if (h1 == h) m += (tm.identity ? 1.f : 0.f) + (tm.qdd ? ldw<E>(tm.qdd, tok * H + hbase + h) : 0.f);
      if (tm.qmat) m += ldw<E>(tm.qmat, (tok * H + hbase + h) * HPG + h1);
      const float *w1 = rec + (set * 2 + 0) * BM * HPG * R + i * HPG * R;
      const float *w2 = rec + (set * 2 + 1) * BM * HPG * R + i * HPG * R;
#pragma unroll
      for (int r = 0; r < R; ++r) m = fmaf(w1[h1 * R + r], w2[r * HPG + h], m);
    }
    (set ? Mpost : Mpre)[(i * HPG + h1) * HPG + h] = m;
  }

  // ---- rows x staged K/V rows of one head: out[(h, i)][j] = f * sum_d A[(h, i)][d] KV[j][d]
  // (the pad rows after the span are rewritten with zeros every time: the
  // region also holds dM between the head loops)
  auto stage = [&](const E *src, int h) {
    for (int idx = tid; idx < (rup(span, 16) + 16) * (D / 8); idx += NT) {
      const int j = idx / (D / 8), ch = idx % (D / 8), s = k_lo + j;
      uint4 u = make_uint4(0, 0, 0, 0);
      if (j < span && s >= 0 && s < T) u = *reinterpret_cast<const uint4 *>(src + row(s, h) + ch * 8);
      *reinterpret_cast<uint4 *>(KVs + j * DP + ch * 8) = u;
    }
  };
  // out[(h, i)][j] = f * sum_d A[(h, i)][d] KV[j][d] on the tensor cores:
  // M = keys (16 per tile, A operand = KV rows), N = queries (8 per tile,
  // B operand = rows of A), K = d
  auto rows_x_kv = [&](const E *A, float *out, int h, float f) {
    const int nmt = (span + 15) / 16, nnt = (BM + 7) / 8;
    const int g8 = lane >> 2, t4 = lane & 3;
    for (int tile = warp; tile < nmt * nnt; tile += NT / 32) {
      const int mt = tile % nmt, nt = tile / nmt;
      float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t af[4], bf[2];
        ldsm_x4(af, KVs + (mt * 16 + (lane & 15)) * DP + ks * 16 + (lane >> 4) * 8);
        ldsm_x2(bf, A + (h * BM + nt * 8 + (lane & 7)) * DP + ks * 16 + ((lane >> 3) & 1) * 8);
        mma16816<E>(c, af, bf);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = mt * 16 + g8 + (e >> 1) * 8, i = nt * 8 + 2 * t4 + (e & 1);
        if (j < span && i < BM) out[(h * BM + i) * SP + j] = f * c[e];
      }
    }
  };
  // dst[s_j][d] += f * sum_i X[(h, i)][j] Y[(h, i)][d] over the block's queries
  // (dV with X = P', Y = dO; dK with X = dL, Y = Q): M = keys, N = d, K = queries
  auto kv_grad = [&](const float *X, const E *Y, float *dst, int h, float f) {
    const int nmt = (span + 15) / 16, nks = (BM + 15) / 16;
    const int g8 = lane >> 2, t4 = lane & 3;
    for (int tile = warp; tile < nmt * (D / 8); tile += NT / 32) {
      const int mt = tile % nmt, nt = tile / nmt;
      float c[4] = {0.f, 0.f, 0.f, 0.f};
      for (int ks = 0; ks < nks; ++ks) {
        uint32_t af[4], bf[2];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int j = mt * 16 + g8 + (r & 1) * 8, i = ks * 16 + 2 * t4 + (r >> 1) * 8;
          const float x0 = i < BM ? X[(h * BM + i) * SP + j] : 0.f;
          const float x1 = i + 1 < BM ? X[(h * BM + i + 1) * SP + j] : 0.f;
          af[r] = pack2<E>(x0, x1);
        }
        ldsm_x2_t(bf, Y + (h * BM + ks * 16 + (lane & 15)) * DP + nt * 8);
        mma16816<E>(c, af, bf);
      }
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int j = mt * 16 + g8 + half * 8, s = k_lo + j;
        if (j < span && s >= 0 && s < T)
          red_add_v2(dst + row(s, h) + nt * 8 + 2 * t4, f * c[2 * half], f * c[2 * half + 1]);
      }
    }
  };
  // per key j, mix the HPG values of query i: dst[(h, i)][j] = sum_h' M[i][h'][h] src[(h', i)][j]
  // (transposed: dst[(h', i)][j] = sum_h M[i][h'][h] src[(h, i)][j])
  // (a task is one key of one query and OC of its outputs; in-place use needs
  // OC == HPG so that a task reads every input before it writes)
  auto mix = [&](const float *M, const float *src, float *dst, bool transposed, bool mask) {
    constexpr int OC = HPG < 8 ? HPG : 8;
    const int noc = (src == dst) ? 1 : HPG / OC;
    for (int idx = tid; idx < BM * SPR * noc; idx += NT) {
      const int j = idx % SPR, i = (idx / SPR) % BM, o0 = (idx / (SPR * BM)) * (noc > 1 ? OC : 0);
      const int o1 = noc > 1 ? o0 + OC : HPG;
      if (j >= span) continue;
      float a[HPG];
#pragma unroll
      for (int h = 0; h < HPG; ++h) a[h] = src[(h * BM + i) * SP + j];
      const bool ok = !mask || valid(q0 + i, k_lo + j);
      const float *Mi = M + i * HPG * HPG;
#pragma unroll 4
      for (int o = o0; o < o1; ++o) {
        float x = 0.f;
#pragma unroll
        for (int k = 0; k < HPG; ++k) x = fmaf(transposed ? Mi[o * HPG + k] : Mi[k * HPG + o], a[k], x);
        dst[(o * BM + i) * SP + j] = ok ? x : -INFINITY;
      }
    }
  };
  // dM[i][h'][h] = sum_j X[(h', i)][j] Y[(h, i)][j], then the weight gradients of one term set
  auto grad_m = [&](const float *X, const float *Y, int set) {
    // one warp per entry, lanes along the keys (contiguous, conflict-free)
    for (int idx = warp; idx < BM * HPG * HPG; idx += NT / 32) {
      const int i = idx / (HPG * HPG), h1 = (idx / HPG) % HPG, h = idx % HPG;
      const float *x = X + (h1 * BM + i) * SP, *y = Y + (h * BM + i) * SP;
      float acc = 0.f;
      for (int j = lane; j < span; j += 32) acc = fmaf(x[j], y[j], acc);
#pragma unroll
      for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) dM[idx] = acc;
    }
    __syncthreads();
    const TermG &gr = set ? p.gpost : p.gpre;
    for (int idx = tid; idx < BM * HPG; idx += NT) {
      const int i = idx / HPG, h = idx % HPG, t = q0 + i;
      if (t >= T) continue;
      const int64_t tok = (int64_t)b * T + t;
      const float *Mi = dM + i * HPG * HPG;
      if (gr.qdd) gr.qdd[tok * H + hbase + h] = Mi[h * HPG + h];
      if (gr.qmat)
        for (int h1 = 0; h1 < HPG; ++h1) gr.qmat[(tok * H + hbase + h) * HPG + h1] = Mi[h1 * HPG + h];
      const float *w1 = rec + (set * 2 + 0) * BM * HPG * R + i * HPG * R;
      const float *w2 = rec + (set * 2 + 1) * BM * HPG * R + i * HPG * R;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (gr.qw1) {  // dqw1[t][h][r] = sum_h2 dM[h][h2] qw2[r][h2]
          float a = 0.f;
          for (int h2 = 0; h2 < HPG; ++h2) a = fmaf(Mi[h * HPG + h2], w2[r * HPG + h2], a);
          gr.qw1[(tok * H + hbase + h) * R + r] = a;
        }
        if (gr.qw2) {  // dqw2[t][r][h] = sum_h1 qw1[h1][r] dM[h1][h]
          float a = 0.f;
          for (int h1 = 0; h1 < HPG; ++h1) a = fmaf(w1[h1 * R + r], Mi[h1 * HPG + h], a);
          gr.qw2[(tok * R + r) * H + hbase + h] = a;
        }
      }
    }
    if (gr.w)
      for (int idx = tid; idx < HPG * HPG; idx += NT) {
        float a = 0.f;
        for (int i = 0; i < BM; ++i)
          if (q0 + i < T) a += dM[i * HPG * HPG + idx];
        atomicAdd(gr.w + (int64_t)g * HPG * HPG + idx, a);
      }
    __syncthreads();
  };

  // ---- L = scale Q K^T (per head), S = pre-mix of L, masked
  for (int h = 0; h < HPG; ++h) {
    __syncthreads();
    stage(kg, h);
    __syncthreads();
    rows_x_kv(Qs, Lb, h, p.scale);
  }
  __syncthreads();
  mix(Mpre, Lb, Pb, false, true);
  __syncthreads();
  // ---- softmax rows (one warp per row); a fully masked row gives P = 0
  for (int c = warp; c < NC; c += NT / 32) {
    float *r = Pb + c * SP;
    float m = -INFINITY;
    for (int j = lane; j < span; j += 32) m = fmaxf(m, r[j]);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    if (m != -INFINITY)
      for (int j = lane; j < span; j += 32) l += __expf(r[j] - m);
#pragma unroll
    for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    const float il = l > 0.f ? 1.f / l : 0.f;
    for (int j = lane; j < span; j += 32) r[j] = m == -INFINITY ? 0.f : __expf(r[j] - m) * il;
  }
  __syncthreads();
  // ---- P' = post-mix of P
  mix(Mpost, Pb, Db, false, false);
  // ---- per head: dV += P'^T dO, then dP' = dO V^T over P'
  for (int h = 0; h < HPG; ++h) {
    __syncthreads();
    kv_grad(Db, dOs, p.dv, h, 1.f);
    stage(vg, h);
    __syncthreads();
    rows_x_kv(dOs, Db, h, 1.f);
  }
  __syncthreads();
  // ---- post set: dMpost = P x dP'
  grad_m(Pb, Db, 1);
  // ---- dP = Mpost^T dP' (in place per key: each task reads all heads first)
  mix(Mpost, Db, Db, true, false);
  __syncthreads();
  // ---- row deltas and dS = P (dP - delta)
  for (int c = warp; c < NC; c += NT / 32) {
    const float *pr = Pb + c * SP, *dr = Db + c * SP;
    float a = 0.f;
    for (int j = lane; j < span; j += 32) a = fmaf(pr[j], dr[j], a);
#pragma unroll
    for (int o = 16; o; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    for (int j = lane; j < span; j += 32) Db[c * SP + j] = pr[j] * (dr[j] - a);
  }
  __syncthreads();
  // ---- pre set: dMpre = L x dS; dL = Mpre^T dS
  grad_m(Lb, Db, 0);
  mix(Mpre, Db, Lb, true, false);
  // ---- per head: dQ = scale dL K, dK += scale dL^T Q
  for (int h = 0; h < HPG; ++h) {
    __syncthreads();
    stage(kg, h);
    __syncthreads();
    // dQ_h[i][d] = scale * sum_j dL[(h, i)][j] K[j][d]: M = queries, N = d, K = keys
    {
      const int nmt = (BM + 15) / 16, nks = (span + 15) / 16;
      const int g8 = lane >> 2, t4 = lane & 3;
      E *dq = reinterpret_cast<E *>(p.dq);
      for (int tile = warp; tile < nmt * (D / 8); tile += NT / 32) {
        const int mt = tile % nmt, nt = tile / nmt;
        float c[4] = {0.f, 0.f, 0.f, 0.f};
        for (int ks = 0; ks < nks; ++ks) {
          uint32_t af[4], bf[2];
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const int i = mt * 16 + g8 + (r & 1) * 8, j = ks * 16 + 2 * t4 + (r >> 1) * 8;
            const float* lr = Lb + (h * BM + i) * SP;
            const float x0 = (i < BM && j < span) ? lr[j] : 0.f;
            const float x1 = (i < BM && j + 1 < span) ? lr[j + 1] : 0.f;
            af[r] = pack2<E>(x0, x1);
          }
          ldsm_x2_t(bf, KVs + (ks * 16 + (lane & 15)) * DP + nt * 8);
          mma16816<E>(c, af, bf);
        }
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int i = mt * 16 + g8 + half * 8, t = q0 + i;
          if (i < BM && t < T)
            *reinterpret_cast<uint32_t *>(dq + row(t, h) + nt * 8 + 2 * t4) =
                pack2<E>(p.scale * c[2 * half], p.scale * c[2 * half + 1]);
        }
      }
    }
    kv_grad(Lb, Qs, p.dk, h, p.scale);
  }
}

template <typename E, int HPG, int R>
static cudaError_t launch_t(const BwdParams &p, cudaStream_t st, std::string *why) {
  const int esize = 2;
  int BM = 64 / HPG > 0 ? 64 / HPG : 1;
  Geo geo = make_geo<HPG, R>(BM, p.window, esize);
  while (geo.total > MAX_SMEM && BM > 1) {
    BM = BM > 1 ? BM / 2 : 1;
    geo = make_geo<HPG, R>(BM, p.window, esize);
  }
  if (geo.total > MAX_SMEM) {
    if (why) *why = "the key span of one query block does not fit in shared memory (window too long)";
    return cudaErrorInvalidValue;
  }
  auto kern = dc_bwd_kernel<E, HPG, R>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, geo.total);
  if (e != cudaSuccess) return e;
  dim3 grid((p.T + BM - 1) / BM, p.B * p.G);
  kern<<<grid, NT, geo.total, st>>>(p, geo);
  return cudaGetLastError();
}

template <typename E, int HPG>
static cudaError_t launch_h(const BwdParams &p, cudaStream_t st, std::string *why) {
  return p.R <= 1 ? launch_t<E, HPG, 1>(p, st, why) : launch_t<E, HPG, 2>(p, st, why);
}

template <typename E>
static cudaError_t launch_e(const BwdParams &p, cudaStream_t st, std::string *why) {
  switch (p.H / p.G) {
    case 1: return launch_h<E, 1>(p, st, why);
    case 2: return launch_h<E, 2>(p, st, why);
    case 4: return launch_h<E, 4>(p, st, why);
    case 8: return launch_h<E, 8>(p, st, why);
    case 16: return launch_h<E, 16>(p, st, why);
    default: return launch_h<E, 32>(p, st, why);
  }
}

}  // namespace bwd

bool bwd_supports(const dc_attn_params &p, std::string *why) {
  auto no = [&](const char *m) { if (why) *why = m; return false; };
  if (p.D != 128) return no("D must be 128");
  const int hpg = p.G > 0 ? p.H / p.G : 0;
  if (hpg != 1 && hpg != 2 && hpg != 4 && hpg != 8 && hpg != 16 && hpg != 32)
    return no("heads per group must be 1, 2, 4, 8, 16 or 32");
  if (p.R > 2) return no("rank R > 2");
  for (const dc_terms *t : {&p.pre, &p.post})
    if (t->kw1 || t->kw2 || t->kdd) return no("the backward does not cover key-wise terms (kw1, kw2, kdd)");
  auto al = [](const void *x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
  if (!al(p.q) || !al(p.k) || !al(p.v)) return no("q, k, v must be 16-byte aligned");
  return true;
}

cudaError_t launch_bwd(const dc_attn_bwd_params &bp, cudaStream_t st, std::string *why) {
  const dc_attn_params &f = bp.fwd;
  bwd::BwdParams p;
  p.B = f.B; p.T = f.T; p.H = f.H; p.G = f.G; p.R = f.R < 1 ? 1 : f.R;
  p.window = f.window > 0 ? (f.window < f.T ? f.window : f.T) : f.T;
  p.scale = f.scale;
  p.q = f.q; p.k = f.k; p.v = f.v; p.dout = bp.dout;
  p.seq_lens = f.seq_lens;
  p.dq = bp.dq; p.dk = bp.dk; p.dv = bp.dv;
  p.pre = to_dev(f.pre); p.post = to_dev(f.post);
  p.gpre = {bp.dpre.w, bp.dpre.qw1, bp.dpre.qw2, bp.dpre.qdd, bp.dpre.qmat};
  p.gpost = {bp.dpost.w, bp.dpost.qw1, bp.dpost.qw2, bp.dpost.qdd, bp.dpost.qmat};
  const size_t n = (size_t)f.B * f.T * f.H * f.D * sizeof(float);
  cudaError_t e = cudaMemsetAsync(bp.dk, 0, n, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(bp.dv, 0, n, st);
  const size_t nw = (size_t)f.H * (f.H / f.G) * sizeof(float);  // G * HPG * HPG
  if (e == cudaSuccess && bp.dpre.w) e = cudaMemsetAsync(bp.dpre.w, 0, nw, st);
  if (e == cudaSuccess && bp.dpost.w) e = cudaMemsetAsync(bp.dpost.w, 0, nw, st);
  if (e != cudaSuccess) return e;
  if (f.dtype == DC_DTYPE_BF16) return bwd::launch_e<__nv_bfloat16>(p, st, why);
  return bwd::launch_e<__half>(p, st, why);
}

}  // namespace dcattn
