// Tensor-core DC-attention forward for windowed layers (sm_100a: TMA, tcgen05, TMEM).
//
// One CTA owns (query block of BM queries, batch b, head group g) for all
// HPG heads of the group, BM * HPG = 128.  The block's key span
// [q0 + BM - 128*NKT, q0 + BM) is cut into NKT key tiles of 128 keys.
//
// Layout choice: keys on TMEM lanes, (head, query) pairs on TMEM columns.
//   S^T_h = K_h Q_h^T     A = K tile [128 keys x D]  (K-major, TMA 128B swizzle)
//                         B = Q_h    [BM x D]        (K-major, TMA 128B swizzle)
//                         D = TMEM lanes = keys, columns kt*128 + h*BM + i
//   O^T_h = V_h^T P'^T_h  A = V tile [128 keys x D]  (MN-major: d contiguous)
//                         B = P'_h   [keys x BM]     (MN-major, written by threads)
//                         D = TMEM lanes = d, columns 128*NKT + h*BM + i
// so one thread (= one key) holds the logits of every head and query of the
// block at its key: the cross-head composition of DC attention
// (dc_attention_torch.py:217-225 and :240-248) is thread-local, and the
// softmax over keys is a cross-lane reduction (redux.sync.max for the max,
// a shuffle transpose-reduce for the sum) plus a cross-warp pass in SMEM.
//
// Warp roles: warps 0 .. 4*NKT-1 compose (warp w: key tile w/4, TMEM lane
// quarter w%4); the last warp's lane 0 issues TMA loads and tcgen05.mma.
// Phases: QK (all heads, all key tiles) -> pre-compose + mask + max ->
// exp + sum -> normalise + post-compose -> P' to SMEM -> PV -> epilogue.
// Every mbarrier wait is bounded; on timeout the kernel records an error code
// in err_flag and skips the remaining work instead of hanging.

#include <cuda.h>
#include <cuda_runtime.h>

#include <string>

#include "tc_common.cuh"

namespace dcattn {
namespace tc {
// F8: q and k are e4m3 (8-bit float) with their scales folded into p.scale;
// QK^T runs as kind::f8f6f4 MMAs, everything else is unchanged.
template <typename E, int HPG, int R, int CS, int MAXT, bool F8 = false>
__global__ void __launch_bounds__(MAXT, 1)
    dc_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_kl,
                 const __grid_constant__ CUtensorMap tm_vl, const __grid_constant__ CUtensorMap tm_o,
                 const TcParams p, const int nkt, const int rlast) {
  constexpr int BM = NQ / HPG;
  constexpr int GI = 32 / HPG;  // queries per 32-value group
  constexpr int NG = BM / GI;   // groups per key tile (= 4)
  static_assert(NG == 4 && NG % CS == 0, "group geometry");

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                          ~static_cast<uintptr_t>(1023));
  const Geo geo = make_geo(HPG, R, nkt);
  float *red = reinterpret_cast<float *>(smem + geo.red_off);    // [2][4*nkt][NQ]
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + geo.bar_off);
  uint64_t *bar_q = bars + 0, *bar_full = bars + 1, *bar_free = bars + 4;
  uint64_t *bar_S = bars + 7 /* [3] */, *bar_P = bars + 10, *bar_O = bars + 11;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + geo.tmem_off);

  const int ncompose_warps = 4 * nkt * CS;
  const int ncompose = 32 * ncompose_warps;
  const int ctrl_warp = ncompose_warps;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.y / p.G, g = blockIdx.y % p.G;
  const int q0 = blockIdx.x * BM;
  const int H = p.H, T = p.T, hbase = g * HPG;
  // key span of the block: [q0 - window + 1, q0 + BM); tile kt covers
  // [kb + 128 kt, kb + 128 kt + 128), the last tile only its first rlast rows
  const int kb = q0 - p.window + 1;
  const int slen = p.seq_lens ? min(max(p.seq_lens[b], 0), T) : T;

  if (threadIdx.x == 0) {
    ptx::mbar_init(bar_q, 1);
    for (int i = 0; i < 3; ++i) {
      ptx::mbar_init(bar_full + i, 1);
      ptx::mbar_init(bar_free + i, 1);
      ptx::mbar_init(bar_S + i, 1);
    }
    ptx::mbar_init(bar_P, ncompose_warps);
    ptx::mbar_init(bar_O, 1);
    ptx::fence_mbar_init();
  }
  if (warp == ctrl_warp) ptx::tmem_alloc(tmem_slot, 512);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t o_col = KT_ROWS * nkt;

  if (warp == ctrl_warp) {
    // ================================================= TMA producer (one thread)
    if (lane == 0 && !p.skip_loads) {
      const int nslot = geo.nslot;
      const int nK = HPG * nkt, total = 2 * nK;
      ptx::tma_prefetch_desc(&tm_q);
      ptx::tma_prefetch_desc(&tm_k);
      ptx::tma_prefetch_desc(&tm_v);
      // Q for every head of the group: two 64-column halves of [BM x 64]
      if constexpr (F8) {  // one 128-byte row per query and head: [head][BM][128 d]
        ptx::mbar_expect_tx(bar_q, NQ * 128);
        for (int h = 0; h < HPG; ++h)
          ptx::tma_load_4d(smem + geo.q_off + h * BM * 128, &tm_q, bar_q, 0, hbase + h, q0, b);
      } else {
        ptx::mbar_expect_tx(bar_q, NQ * 256);
        for (int h = 0; h < HPG; ++h)
          for (int c = 0; c < 2; ++c)
            ptx::tma_load_4d(smem + geo.q_off + h * BM * 256 + c * BM * 128, &tm_q, bar_q, c * 64, hbase + h, q0, b);
      }
      // jobs are key-tile major: job j -> key tile j / HPG, head j % HPG; K jobs then V jobs
      for (int j = 0; j < total; ++j) {
        const int slot = j % nslot, use = j / nslot;
        if (use > 0 && !ptx::mbar_wait(bar_free + slot, (use - 1) & 1, p.wait_us)) {
          record_err(p, ERR_TIMEOUT_FREE);
          break;
        }
        const bool isv = j >= nK;
        const int jj = j % nK, kt = jj / HPG, h = jj % HPG;
        const bool last = kt == nkt - 1;
        const CUtensorMap *m = isv ? (last ? &tm_vl : &tm_v) : (last ? &tm_kl : &tm_k);
        const int rows = last ? rlast : KT_ROWS;
        unsigned char *dst = smem + geo.ring_off + slot * TILE_BYTES;
        if (F8 && !isv) {  // an e4m3 K tile: one box of 128-byte rows
          ptx::mbar_expect_tx(bar_full + slot, rows * 128);
          ptx::tma_load_4d(dst, m, bar_full + slot, 0, hbase + h, kb + kt * KT_ROWS, b);
        } else {
          ptx::mbar_expect_tx(bar_full + slot, rows * 256);
          ptx::tma_load_4d(dst, m, bar_full + slot, 0, hbase + h, kb + kt * KT_ROWS, b);
          ptx::tma_load_4d(dst + TILE_BYTES / 2, m, bar_full + slot, 64, hbase + h, kb + kt * KT_ROWS, b);
        }
      }
    }
    __syncwarp();
  } else if (warp == ctrl_warp + 1) {
    // ================================================= MMA issuer
    // Whole warp runs the loops; one elected lane issues each tcgen05 op.
    const uint32_t ab_fmt = std::is_same<E, __nv_bfloat16>::value ? 1u : 0u;
    const uint32_t idesc_qk = ptx::idesc_f16(ab_fmt, 0, 0, 128, BM);
    const uint32_t idesc_pv = ptx::idesc_f16(ab_fmt, 1, 1, 128, BM);
    const uint64_t qd0 = ptx::smem_desc(ptx::smem_u32(smem + geo.q_off), 16, 1024, 2);
    const uint64_t kd0 = ptx::smem_desc(ptx::smem_u32(smem + geo.ring_off), 16, 1024, 2);
    // V tile, MN-major 128B swizzle: 8-key groups 1024 B apart, d halves 16 KB apart
    const uint64_t vd0 = ptx::smem_desc(ptx::smem_u32(smem + geo.ring_off), TILE_BYTES / 2, 1024, 2);
    // P' tile, MN-major no swizzle: 8x8 core matrices, query blocks 128 B apart,
    // 8-key blocks BM*16 B apart
    const uint64_t pd0 = ptx::smem_desc(ptx::smem_u32(smem + geo.p_off), BM * 16, 128, 0);
    const int nslot = geo.nslot;
    const int nK = HPG * nkt, total = 2 * nK;
    bool ok = true;
    auto wait_u = [&](uint64_t *bar, int parity, int code) {
      const bool got = __all_sync(0xffffffffu, ok && ptx::mbar_wait(bar, parity, p.wait_us));
      if (ok && !got) {
        ok = false;
        if (lane == 0) record_err(p, code);
      }
      return ok;
    };
    wait_u(bar_q, 0, ERR_TIMEOUT_Q);
    // ---- S^T_h = K_h Q_h^T; key tile kt is signalled as soon as its heads are issued
    for (int j = 0; j < nK && ok; ++j) {
      const int slot = j % nslot;
      if (!wait_u(bar_full + slot, (j / nslot) & 1, ERR_TIMEOUT_FULL)) break;
      ptx::tc_fence_after();
      const int kt = j / HPG, h = j % HPG;
      const uint64_t ad = ptx::desc_add(kd0, slot * TILE_BYTES);
      const uint32_t dd = tbase + kt * KT_ROWS + h * BM;
      if constexpr (F8) {
        // 32 e4m3 elements (32 bytes) per K step: four steps along one 128-byte row
        const uint64_t bd = ptx::desc_add(qd0, h * BM * 128);
        const uint32_t idesc_qk8 = ptx::idesc_f16(0, 0, 0, 128, BM);  // e4m3 x e4m3 -> f32
#pragma unroll
        for (int ks = 0; ks < D / 32; ++ks)
          if (ptx::elect_one())
            ptx::mma_f8_ss(dd, ptx::desc_add(ad, ks * 32), ptx::desc_add(bd, ks * 32), idesc_qk8, ks > 0);
      } else {
        const uint64_t bd = ptx::desc_add(qd0, h * BM * 256);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          if (ptx::elect_one())
            ptx::mma_f16_ss(dd, ptx::desc_add(ad, (ks >> 2) * (TILE_BYTES / 2) + (ks & 3) * 32),
                            ptx::desc_add(bd, (ks >> 2) * (BM * 128) + (ks & 3) * 32), idesc_qk, ks > 0);
      }
      if (ptx::elect_one()) {
        ptx::mma_commit(bar_free + slot);
        if (h == HPG - 1) ptx::mma_commit(bar_S + kt);
      }
      __syncwarp();
    }
    // ---- O^T_h = V_h^T P'^T_h, accumulated over key tiles
    if (ok) wait_u(bar_P, 0, ERR_TIMEOUT_P);
    ptx::tc_fence_after();
    for (int j = nK; j < total && ok; ++j) {
      const int slot = j % nslot;
      if (!wait_u(bar_full + slot, (j / nslot) & 1, ERR_TIMEOUT_FULL)) break;
      ptx::tc_fence_after();
      const int jj = j - nK, kt = jj / HPG, h = jj % HPG;
      const int ksteps = (kt == nkt - 1 ? rlast : KT_ROWS) / 16;
      const uint64_t ad = ptx::desc_add(vd0, slot * TILE_BYTES);
      const uint64_t bd = ptx::desc_add(pd0, (h * nkt + kt) * (KT_ROWS * BM * 2));
      const uint32_t dd = tbase + o_col + h * BM;
#pragma unroll
      for (int ks = 0; ks < KT_ROWS / 16; ++ks)
        if (ks < ksteps && ptx::elect_one())
          ptx::mma_f16_ss(dd, ptx::desc_add(ad, ks * 2048), ptx::desc_add(bd, ks * (2 * BM * 16)), idesc_pv,
                          (kt > 0 || ks > 0));
      if (ptx::elect_one()) ptx::mma_commit(bar_free + slot);
      __syncwarp();
    }
    if (ptx::elect_one()) ptx::mma_commit(bar_O);
    __syncwarp();
  } else {
    // ================================================= compose warps
    // Composition as in dc_tcp_kernel: per-query mixing matrices M_t (every
    // query-dependent term of a set folded into one HPG x HPG matrix, the pre
    // set scaled by scale * log2(e)), key weights in registers, two queries per
    // paired-fp32 instruction at 1-4 heads per group, fixed-point warp sums.
    constexpr bool PAIR = HPG <= 4;
    constexpr int RAWF = HPG * (2 * R + 1), MF = HPG * HPG, NCK = 2 * R + 1, NCH = 2 * BM * NCK;
    float *raw = reinterpret_cast<float *>(smem + geo.rec_off);    // [set][BM][RAWF]
    float *mrec = reinterpret_cast<float *>(smem + geo.mrec_off);  // [set][BM][h'][h] (pair layout with PAIR)
    float *redm = red;                                             // [4*nkt][NQ] column maxima (base 2)
    uint32_t *reds = reinterpret_cast<uint32_t *>(red + 4 * nkt * NQ);  // [4*nkt][NQ] fixed-point sums
    float *fac = reinterpret_cast<float *>(smem + geo.fac_off);    // [4*nkt][BM][HPG] (pair layout with PAIR)
    const float sl2e = p.scale * kLog2e;
    // per-query weights of the block in chunks of HPG contiguous elements:
    // chunk (set, query i, k), k = 0: qdd; 1..R: qw1 [h][r]; R+1..2R: qw2 [r][h]
    for (int c = threadIdx.x; c < NCH; c += ncompose) {
      const int set = c / (BM * NCK), rem = c % (BM * NCK), i = rem / NCK, k = rem % NCK;
      const TermPtrs &tm = set ? p.post : p.pre;
      const int t = q0 + i;
      const int64_t tok = (int64_t)b * T + t;
      const E *src = nullptr;
      if (t < T) {
        if (k == 0) src = tm.qdd ? elem<E>(tm.qdd, tok * H + hbase) : nullptr;
        else if (k <= R) src = tm.qw1 ? elem<E>(tm.qw1, (tok * H + hbase) * R + (k - 1) * HPG) : nullptr;
        else src = tm.qw2 ? elem<E>(tm.qw2, (tok * R + (k - 1 - R)) * H + hbase) : nullptr;
      }
      const Raw16<HPG> v = src ? ld_raw16<HPG>(src) : raw16_zero<HPG>();
      float *dst = raw + (set * BM + i) * RAWF + k * HPG;
#pragma unroll
      for (int h = 0; h < HPG; ++h) dst[h] = raw16_get<E, HPG>(v, h);
    }
    // warp -> (lane quarter sub, key tile kt, column half cs); warps sharing
    // (sub, kt) split the NG column groups of the tile between them
    const int sub = warp & 3, kt = (warp >> 2) % nkt, cs = warp / (4 * nkt);
    const int rw = warp % (4 * nkt);  // reduction slot: one writer per (column, sub, kt)
    const int g_begin = cs * (NG / CS), g_end = g_begin + NG / CS;
    const int s_local = 32 * sub + lane;          // key row inside the key tile
    const int s = kb + kt * KT_ROWS + s_local;    // absolute key index
    const bool key_ok = s >= 0 && s < slen;
    const uint32_t tl = tbase + (static_cast<uint32_t>(32 * sub) << 16) + kt * KT_ROWS;
    const int wk0 = kb + kt * KT_ROWS + 32 * sub;
    const int klo = max(0, kb), khi = min(q0 + BM - 1, slen - 1);
    const bool active = wk0 + 31 >= klo && wk0 <= khi;
    const int64_t ktok = (int64_t)b * T + s;
    const bool keys_in = wk0 >= 0 && wk0 + 31 < slen;
    auto all_valid = [&](int t0) {
      return keys_in && wk0 + 31 <= t0 && t0 + GI - 1 - wk0 < p.window && t0 + GI - 1 < T;
    };
    auto valid = [&](int t) { return key_ok && s <= t && t - s < p.window && t < T; };
    bool ok = true;

    float kw1[HPG * R], kw2[R * HPG], kdd[HPG];
    ptx::f2_t kw1d[HPG * R], kw2d[R * HPG], kddd[HPG];
    auto load_key = [&](const TermPtrs &tm, float f) {
      load_key_weights_vec<E, HPG, R>(tm, ktok, H, hbase, key_ok && active, kw1, kw2, kdd);
#pragma unroll
      for (int j = 0; j < R * HPG; ++j) kw2[j] *= f;
#pragma unroll
      for (int j = 0; j < HPG; ++j) kdd[j] *= f;
      if constexpr (PAIR) {
#pragma unroll
        for (int j = 0; j < HPG * R; ++j) kw1d[j] = ptx::f2_dup(kw1[j]);
#pragma unroll
        for (int j = 0; j < R * HPG; ++j) kw2d[j] = ptx::f2_dup(kw2[j]);
#pragma unroll
        for (int j = 0; j < HPG; ++j) kddd[j] = ptx::f2_dup(kdd[j]);
      }
    };
    load_key(p.pre, sl2e);
    ptx::named_bar_sync(1, ncompose);  // per-query weights staged
    for (int idx = threadIdx.x; idx < 2 * BM * MF; idx += ncompose) {
      const int set = idx / (BM * MF), i = (idx / MF) % BM, h1 = (idx % MF) / HPG, h = idx % HPG;
      const TermPtrs &tm = set ? p.post : p.pre;
      const float *rr = raw + (set * BM + i) * RAWF;
      float m = (tm.w ? tm.w[((int64_t)g * HPG + h1) * HPG + h] : 0.f) + (h1 == h ? (tm.identity ? 1.f : 0.f) + rr[h] : 0.f) +
                qmat_at<E>(tm, b, q0 + i, T, H, HPG, hbase, h1, h);
#pragma unroll
      for (int r = 0; r < R; ++r) m = fmaf(rr[HPG + h1 * R + r], rr[HPG + HPG * R + r * HPG + h], m);
      mrec[PAIR ? set * BM * MF + (i >> 1) * 2 * MF + (h1 * HPG + h) * 2 + (i & 1) : idx] = set ? m : m * sl2e;
    }
    ptx::named_bar_sync(1, ncompose);  // matrices visible
    if (!ptx::mbar_wait(bar_S + kt, 0, p.wait_us)) { ok = false; record_err(p, ERR_TIMEOUT_S); }
    ptx::tc_fence_after();

    // ---- pass 1: pre-composition (+ mask at the window's edges), warp-local column max,
    //      e = 2^(S - m_w) back to TMEM, fixed-point warp-local column sums
#pragma unroll 1
    for (int grp = g_begin; grp < g_end; ++grp) {
      const int i0 = grp * GI;
      float *mx = redm + rw * NQ + i0;
      uint32_t *sx = reds + rw * NQ + i0;
      if (active && ok) {
        float v[HPG][GI];
#pragma unroll
        for (int h = 0; h < HPG; ++h) ptx::tmem_ld<GI>(tl + h * BM + i0, v[h]);
        ptx::tmem_wait_ld();
        const bool full = all_valid(q0 + i0);
        if constexpr (PAIR) {
#pragma unroll
          for (int ii = 0; ii < GI; ii += 2) {
            ptx::f2_t a[HPG], o[HPG];
#pragma unroll
            for (int h = 0; h < HPG; ++h) a[h] = ptx::f2_pack(v[h][ii], v[h][ii + 1]);
            compose_m2<HPG, R>(a, o, mrec + (i0 + ii) * MF, kw1d, kw2d, kddd);
            const bool vl0 = full || valid(q0 + i0 + ii), vl1 = full || valid(q0 + i0 + ii + 1);
#pragma unroll
            for (int h = 0; h < HPG; ++h) {
              v[h][ii] = vl0 ? ptx::f2_lo(o[h]) : kMaskedLogit;
              v[h][ii + 1] = vl1 ? ptx::f2_hi(o[h]) : kMaskedLogit;
            }
          }
        } else {
#pragma unroll
          for (int ii = 0; ii < GI; ++ii) {
            float a[HPG], o[HPG];
#pragma unroll
            for (int h = 0; h < HPG; ++h) a[h] = v[h][ii];
            compose_m<HPG, R>(a, o, mrec + (i0 + ii) * MF, kw1, kw2, kdd);
            const bool vl = full || valid(q0 + i0 + ii);
#pragma unroll
            for (int h = 0; h < HPG; ++h) v[h][ii] = vl ? o[h] : kMaskedLogit;
          }
        }
#pragma unroll
        for (int h = 0; h < HPG; ++h) {
          float m8[GI];
          uint32_t s8[GI];
#pragma unroll
          for (int ii = 0; ii < GI; ++ii) {
            m8[ii] = ptx::warp_max(v[h][ii]);
            v[h][ii] = ptx::ex2(v[h][ii] - m8[ii]);
            s8[ii] = ptx::warp_sum_u32(__float_as_uint(v[h][ii] + 1.f));
          }
          if (lane == 0) {
#pragma unroll
            for (int ii = 0; ii < GI; ii += 4) {
              *reinterpret_cast<float4 *>(mx + h * BM + ii) = make_float4(m8[ii], m8[ii + 1], m8[ii + 2], m8[ii + 3]);
              *reinterpret_cast<uint4 *>(sx + h * BM + ii) = make_uint4(s8[ii], s8[ii + 1], s8[ii + 2], s8[ii + 3]);
            }
          }
        }
#pragma unroll
        for (int h = 0; h < HPG; ++h) ptx::tmem_st<GI>(tl + h * BM + i0, v[h]);
      } else if (lane == 0) {
#pragma unroll
        for (int h = 0; h < HPG; ++h)
#pragma unroll
          for (int ii = 0; ii < GI; ii += 4) {
            *reinterpret_cast<float4 *>(mx + h * BM + ii) =
                make_float4(kMaskedLogit, kMaskedLogit, kMaskedLogit, kMaskedLogit);
            *reinterpret_cast<uint4 *>(sx + h * BM + ii) = make_uint4(0u, 0u, 0u, 0u);
          }
      }
    }
    // the post-set key weights replace the pre-set ones (dead after pass 1)
    load_key(p.post, 1.f);
    ptx::tmem_wait_st();
    ptx::named_bar_sync(1, ncompose);
    // combine the slots of each column: m = max_w m_w, l = sum_w sum_w 2^(m_w - m),
    // factor_w = 2^(m_w - m) / l; an all-masked column gets factor 0
    constexpr int MAXSL = 12;  // 4 lane quarters x at most 3 key tiles
    const int nslots = 4 * nkt;
    for (int j = threadIdx.x; j < NQ; j += ncompose) {
      float mw[MAXSL];
      uint32_t sw[MAXSL];
#pragma unroll
      for (int w = 0; w < MAXSL; ++w) {
        mw[w] = w < nslots ? redm[w * NQ + j] : kMaskedLogit;
        sw[w] = w < nslots ? reds[w * NQ + j] : 32u * 0x3F800000u;
      }
      float m = mw[0];
#pragma unroll
      for (int w = 1; w < MAXSL; ++w) m = fmaxf(m, mw[w]);
      float l = 0.f;
#pragma unroll
      for (int w = 0; w < MAXSL; ++w) {
        mw[w] = ptx::ex2(mw[w] - m);
        l = fmaf(mw[w], static_cast<float>(sw[w] - 32u * 0x3F800000u) * 0x1p-23f, l);
      }
      const float il = (m > 0.5f * kMaskedLogit && l > 0.f) ? __frcp_rn(l) : 0.f;
      const int h = j / BM, i = j % BM;
#pragma unroll
      for (int w = 0; w < MAXSL; ++w)
        if (w < nslots)
          fac[w * BM * HPG + (PAIR ? (i >> 1) * 2 * HPG + h * 2 + (i & 1) : i * HPG + h)] = mw[w] * il;
    }
    ptx::named_bar_sync(1, ncompose);

    // ---- pass 2: normalise, post-composition, P' -> SMEM (PV B operand)
    const float *fw = fac + rw * BM * HPG;
    unsigned char *prow = smem + geo.p_off + (s_local & 7) * 16 + (s_local >> 3) * (BM * 16);
#pragma unroll 1
    for (int grp = g_begin; grp < g_end; ++grp) {
      const int i0 = grp * GI;
      float v[HPG][GI];
      if (active && ok) {
#pragma unroll
        for (int h = 0; h < HPG; ++h) ptx::tmem_ld<GI>(tl + h * BM + i0, v[h]);
        ptx::tmem_wait_ld();
        if constexpr (PAIR) {
#pragma unroll
          for (int ii = 0; ii < GI; ii += 2) {
            ptx::f2_t a[HPG], o[HPG];
            float f[2 * HPG];
            ld_row<2 * HPG>(fw + (i0 + ii) * HPG, f);
#pragma unroll
            for (int h = 0; h < HPG; ++h)
              a[h] = ptx::f2_mul(ptx::f2_pack(v[h][ii], v[h][ii + 1]), ptx::f2_pack(f[2 * h], f[2 * h + 1]));
            compose_m2<HPG, R>(a, o, mrec + (BM + i0 + ii) * MF, kw1d, kw2d, kddd);
#pragma unroll
            for (int h = 0; h < HPG; ++h) {
              v[h][ii] = ptx::f2_lo(o[h]);
              v[h][ii + 1] = ptx::f2_hi(o[h]);
            }
          }
        } else {
#pragma unroll
          for (int ii = 0; ii < GI; ++ii) {
            float a[HPG], o[HPG], f[HPG];
            ld_row<HPG>(fw + (i0 + ii) * HPG, f);
#pragma unroll
            for (int h = 0; h < HPG; ++h) a[h] = v[h][ii] * f[h];
            compose_m<HPG, R>(a, o, mrec + (BM + i0 + ii) * MF, kw1, kw2, kdd);
#pragma unroll
            for (int h = 0; h < HPG; ++h) v[h][ii] = o[h];
          }
        }
      } else {
#pragma unroll
        for (int h = 0; h < HPG; ++h)
#pragma unroll
          for (int ii = 0; ii < GI; ++ii) v[h][ii] = 0.f;
      }
#pragma unroll
      for (int h = 0; h < HPG; ++h) {
        unsigned char *tile = prow + (h * nkt + kt) * (KT_ROWS * BM * 2);
#pragma unroll
        for (int c = 0; c < GI; c += 8 < GI ? 8 : GI) {
          // up to 8 queries -> one 16-byte row of an 8x8 core matrix
          constexpr int W8 = GI < 8 ? GI : 8;
          uint32_t pk[W8 / 2];
#pragma unroll
          for (int u = 0; u < W8 / 2; ++u) pk[u] = pack2<E>(v[h][c + 2 * u], v[h][c + 2 * u + 1]);
          const int i = i0 + c;
          unsigned char *dst = tile + (i >> 3) * 128 + (i & 7) * 2;
          if constexpr (W8 == 8) {
            *reinterpret_cast<uint4 *>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          } else if constexpr (W8 == 4) {
            *reinterpret_cast<uint2 *>(dst) = make_uint2(pk[0], pk[1]);
          } else {
            *reinterpret_cast<uint32_t *>(dst) = pk[0];
          }
        }
      }
    }
    ptx::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(bar_P);

    // ---- epilogue: O^T (lanes = d) -> SMEM [head][d half][query][64 d] -> TMA store
    if (!ptx::mbar_wait(bar_O, 0, p.wait_us)) { ok = false; record_err(p, ERR_TIMEOUT_O); }
    ptx::tc_fence_after();
    unsigned char *stage = smem + geo.q_off;  // Q is dead once every MMA has completed
    const int d = 32 * sub + lane;
    if (ok) {
#pragma unroll 1
      for (int c = warp >> 2; c < NQ / 8; c += nkt * CS) {
        float v[8];
        ptx::tmem_ld<8>(tbase + (static_cast<uint32_t>(32 * sub) << 16) + o_col + 8 * c, v);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const int col = 8 * c + jj, h = col / BM, i = col % BM;
          *reinterpret_cast<E *>(stage + (h * 2 + (d >> 6)) * (BM * 128) + i * 128 + (d & 63) * 2) =
              from_f<E>(v[jj]);
        }
      }
    }
    ptx::fence_proxy_async_smem();
    ptx::named_bar_sync(1, ncompose);
    if (threadIdx.x == 0 && ok) {
      for (int h = 0; h < HPG; ++h)
        for (int c = 0; c < 2; ++c)
          ptx::tma_store_4d(&tm_o, stage + (h * 2 + c) * (BM * 128), c * 64, hbase + h, q0, b);
      ptx::bulk_commit();
      ptx::bulk_wait_read0();
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == ctrl_warp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tbase, 512);
  }
}

// ------------------------------------------------------------------ persistent kernel
//
// Windowed layers whose key span fits two key tiles (BM + window - 1 <= 256)
// run persistently: one CTA per SM walks the (query block, batch, group)
// tiles blockIdx.x, blockIdx.x + gridDim.x, ... and overlaps consecutive
// tiles with double buffers:
//   TMEM  two 256-column buffers; buffer = S of both key tiles, and after
//         pass 2 the PV accumulator O aliases key tile 0's columns;
//   SMEM  two Q buffers; a Q buffer becomes P' of key tile 0 once its QK
//         products are done, then the output staging tile of the epilogue;
//         two P' buffers for key tile 1; one K/V ring shared by all tiles.
// Warps: compose warps (as in dc_tc_kernel), 4 epilogue warps (TMEM -> SMEM
// -> TMA store), one TMA warp, one MMA warp.  Order of ring jobs and MMAs:
// Q(n) K(n) V(n-1), i.e. QK(n) is issued before PV(n-1) so the compose warps
// can start tile n while tile n-1 drains.

// Warp-role table of the persistent kernel, built on the host.  Compose warps
// exist only for the TMEM lane quarters that hold keys of their key tile (the
// last key tile is usually short), and a compose warp must sit at an index
// with warp % 4 == its lane quarter (tcgen05.ld / st address the quarter of
// warp % 4), so the other roles fill the gaps.
enum : uint8_t { ROLE_IDLE = 0xFF, ROLE_TMA = 0x80, ROLE_MMA = 0x81, ROLE_EPI = 0x90 /* | quarter */ };
struct WarpRoles {
  uint8_t role[32];  // compose: kt << 3 | cs << 2 | sub
  int nwarps, ncw, nslots, epi_leader;
};

// A second key tile of at most 32 rows would put all its keys in TMEM lane
// quarter 0 and so all its compose warps on one SM sub-partition (a warp reads
// only the lane quarter of its index mod 4), doubling that sub-partition's
// share of the composition.  Instead its K rows are loaded to rows 64 and 96
// of the MMA operand: lane quarters 2 and 3 hold its keys, and one warp in
// each composes half of its columns.  Quarters 0 and 1 are left out because
// their sub-partitions also run the TMA and MMA warps.
// (At 8 heads per group the extra K loads cost more than the balance gains.)
__host__ __device__ inline bool replicated_last(int nkt, int rlast, int hpg) {
  return nkt == 2 && rlast <= 32 && hpg <= 4;
}

static WarpRoles make_roles(int nkt, int rlast, int CS, int hpg) {
  WarpRoles r;
  for (int i = 0; i < 32; ++i) r.role[i] = ROLE_IDLE;
  bool used[32] = {false};
  bool fits = true;  // every role found a warp index below 32
  // first free index at start, start + step, ...; -1 when none is left
  auto free_from = [&](int start, int step) {
    int w = start;
    while (w < 32 && used[w]) w += step;
    if (w >= 32) { fits = false; return -1; }
    used[w] = true;
    return w;
  };
  const bool rep = replicated_last(nkt, rlast, hpg);
  const int nq_last = (rlast + 31) / 32;
  r.ncw = 0;
  for (int kt = 0; kt < nkt; ++kt) {
    const bool rk = rep && kt == nkt - 1;  // one warp in quarters 2 and 3, two column groups each
    const int nq = kt < nkt - 1 || rk ? 4 : nq_last;
    for (int cs = 0; cs < (rk ? 1 : CS); ++cs)
      for (int sub = rk ? 2 : 0; sub < nq; ++sub) {
        const int w = free_from(sub, 4);
        if (w < 0) continue;
        r.role[w] = static_cast<uint8_t>(kt << 3 | cs << 2 | sub);
        ++r.ncw;
      }
  }
  r.nslots = 4 * (nkt - 1) + nq_last;
  auto take = [&](uint8_t role, int quarter) {
    const int w = quarter < 0 ? free_from(0, 1) : free_from(quarter, 4);
    if (w >= 0) r.role[w] = role;
    return w;
  };
  take(ROLE_TMA, -1);
  take(ROLE_MMA, -1);
  r.epi_leader = take(ROLE_EPI | 0, 0);
  for (int q = 1; q < 4; ++q) take(static_cast<uint8_t>(ROLE_EPI | q), q);
  r.nwarps = 0;
  for (int i = 0; i < 32; ++i)
    if (used[i]) r.nwarps = i + 1;
  if (!fits) r.nwarps = 0;  // no valid table: the launcher runs the per-tile kernel
  return r;
}

struct GeoP {
  int nslot, q_off, p1_off, ring_off, wz_off, raw_off, mrec_off, red_off, fac_off, bar_off, tmem_off, stage_off,
      total, raw_floats, p1_bytes;
};

__host__ __device__ inline GeoP make_geo_p(int HPG, int R, int rlast, int nslot, int G) {
  GeoP g{};
  const int BM = NQ / HPG;
  g.nslot = nslot;
  g.q_off = 0;                                   // 2 x (NQ * 256): Q / P'(tile 0) / staging
  g.p1_bytes = round_up(HPG * rlast * BM * 2, 1024);
  g.p1_off = 2 * NQ * 256;                       // 2 x P'(tile 1)
  g.ring_off = g.p1_off + 2 * g.p1_bytes;
  // the short last key tile of all heads may share one slot (see packed_last);
  // the QK MMA then reads 128 rows from each head's half: pad the ring's end
  // (the read-only over-read may run into the data placed after the ring, as
  // long as it stays inside this CTA's shared memory)
  int pad = 0;
  if (HPG > 1 && HPG * rlast * 256 <= TILE_BYTES) pad = (2 * HPG - 1) * rlast * 128 + TILE_BYTES / 2 - TILE_BYTES;
  const int ring_end = g.ring_off + nslot * TILE_BYTES;
  int o = ring_end;
  g.raw_floats = HPG * (2 * R + 1);
  // static mix of every group with the identity on its diagonal [set][G][h'][h]:
  // a persistent CTA's tiles belong to different groups
  g.wz_off = o;  o += 2 * G * HPG * HPG * 4;
  // per-query weights as loaded (qdd[h] | qw1[h][r] | qw2[r][h]) [parity][set][BM]:
  // tile n+1's are fetched during tile n
  g.raw_off = round_up(o, 16); o = g.raw_off + 2 * 2 * BM * g.raw_floats * 4;
  // per-query mixing matrices [parity][set][BM][h'][h]: tile n+1's are built during tile n
  g.mrec_off = round_up(o, 16); o = g.mrec_off + 2 * 2 * BM * HPG * HPG * 4;
  g.red_off = round_up(o, 16); o = g.red_off + 2 * 8 * NQ * 4;   // column maxima | column sums
  g.fac_off = o; o += 8 * NQ * 4;                                 // probability factors [slot][BM][HPG]
  g.bar_off = round_up(o, 8); o = g.bar_off + 32 * 8;
  g.tmem_off = o; o += 16;
  g.stage_off = round_up(o, 1024); o = g.stage_off + 8192;  // epilogue staging (32 columns)
  g.total = o > ring_end + pad ? o : ring_end + pad;
  return g;
}

template <typename E, int HPG, int R, int CS, int NW>
__global__ void __launch_bounds__(32 * NW, 1)
    dc_tcp_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_kl,
                  const __grid_constant__ CUtensorMap tm_vl, const __grid_constant__ CUtensorMap tm_o,
                  const TcParams p, const int nkt, const int rlast, const int nslot, const WarpRoles roles) {
  constexpr int BM = NQ / HPG;
  constexpr int GI = 32 / HPG;
  constexpr int NG = BM / GI;
  // compose two queries per paired-fp32 instruction (compose_m2); at 8 heads
  // per group the duplicated key weights and the wider rows spill, so those
  // groups compose one query at a time
  constexpr bool PAIR = HPG <= 4;
  // build the next tile's matrices inside the statistics window (by the
  // threads that do not combine columns) and run tiles without a barrier
  // between them; at 8 heads per group the larger matrices make that window
  // the longer path, so those build after it and keep the tile barrier
  constexpr bool EARLY_M = HPG <= 4;
  static_assert(NG == 4 && NG % CS == 0, "group geometry");

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                          ~static_cast<uintptr_t>(1023));
  const GeoP geo = make_geo_p(HPG, R, rlast, nslot, p.G);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + geo.bar_off);
  uint64_t *bar_full = bars + 0, *bar_free = bars + 22;         // ring (up to 4 slots each)
  uint64_t *bar_q = bars + 6;                                    // [2] Q landed
  uint64_t *bar_S = bars + 8;                                    // [2][2] S of (buffer, key tile) ready
  uint64_t *bar_P = bars + 12;                                   // [2] P' written (compose warps)
  uint64_t *bar_O = bars + 14;                                   // [2] O complete (PV committed)
  uint64_t *bar_Ofree = bars + 16;                               // [2] O read out of TMEM (epilogue)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + geo.tmem_off);

  const int ncw = roles.ncw;  // compose warps
  const int ncompose = 32 * ncw;
  const int nslots = roles.nslots;  // reduction slots: one per (key tile, lane quarter) with keys
  const int epi_warp0 = roles.epi_leader;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint8_t role = roles.role[warp];
  const int nqb = (p.T + BM - 1) / BM;
  const int ntiles = nqb * p.B * p.G;
  const int H = p.H, T = p.T;
  const int rows_of[2] = {nkt == 1 ? rlast : KT_ROWS, rlast};
  // K/V jobs of one tile: one per (key tile, head) for full key tiles.  The
  // short last key tile is packed: all heads in one job when they fit a slot;
  // when replicated (two copies of its K rows, see replicated_last) two heads
  // per K job, laid out [head][d half][copy][rows] and read by the MMA from
  // 128 - 2 * rlast rows before the copies, so that they land in TMEM lane
  // quarters 2 and 3; its V then fits one packed job.
  const bool rep_last = replicated_last(nkt, rlast, HPG);
  const bool packed_last = !rep_last && HPG > 1 && HPG * rlast * 256 <= TILE_BYTES;
  const int kph = rep_last ? (HPG < 2 ? HPG : 2) : 1;
  const int nlastK = packed_last ? 1 : rep_last ? HPG / kph : HPG;
  const bool vpack = packed_last || (rep_last && HPG > 1 && HPG * rlast * 256 <= TILE_BYTES);
  const int nlastV = vpack ? 1 : HPG;
  const int nfull = HPG * (nkt - 1);
  const int nKk = nfull + nlastK, nKv = nfull + nlastV;
  // half: byte distance of the d halves; aoff: start of the 128-row MMA operand
  // relative to a head's data
  struct Job { int kt, h0, nh, rows, half, ncopy, aoff; };
  // K jobs visit the last key tile first: its compose warps then start with
  // the others instead of one key-tile load later; V jobs keep key-tile order
  // (the first PV product of a tile initialises the accumulator)
  auto job_of = [&](int jj, bool isv) {
    if (!isv && nkt > 1) jj = jj < nlastK ? nfull + jj : jj - nlastK;
    Job j;
    j.ncopy = 1;
    j.aoff = 0;
    if (jj < nfull) {
      j.kt = jj / HPG; j.h0 = jj % HPG; j.nh = 1; j.rows = KT_ROWS; j.half = TILE_BYTES / 2;
    } else {
      const int l = jj - nfull;
      j.kt = nkt - 1;
      j.rows = rows_of[j.kt];
      if (!isv && rep_last) {
        j.nh = kph; j.h0 = l * kph; j.ncopy = 2; j.half = 2 * j.rows * 128;
        j.aoff = -(KT_ROWS - 2 * j.rows) * 128;
      } else if (isv ? vpack : packed_last) {
        j.nh = HPG; j.h0 = 0; j.half = j.rows * 128;
      } else {
        j.nh = 1; j.h0 = l; j.half = TILE_BYTES / 2;
      }
    }
    return j;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 4; ++i) {
      ptx::mbar_init(bar_full + i, 1);
      ptx::mbar_init(bar_free + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(bar_q + i, 1);
      ptx::mbar_init(bar_S + 2 * i, 1);
      ptx::mbar_init(bar_S + 2 * i + 1, 1);
      ptx::mbar_init(bar_P + i, ncw);
      ptx::mbar_init(bar_O + i, 1);
      ptx::mbar_init(bar_Ofree + i, 4);
    }
    ptx::fence_mbar_init();
  }
  if (role == ROLE_TMA) ptx::tmem_alloc(tmem_slot, 512);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t WAIT = p.wait_us;

  // tile -> (query block, batch, group)
  auto tile_coords = [&](int tile, int &q0, int &b, int &g) {
    const int qb = tile % nqb, bg = tile / nqb;
    q0 = qb * BM; b = bg / p.G; g = bg % p.G;
  };
  // P' base of (buffer, key tile)
  auto p_tile = [&](int buf, int kt) -> unsigned char * {
    return kt == 0 ? smem + geo.q_off + buf * NQ * 256 : smem + geo.p1_off + buf * geo.p1_bytes;
  };

  if (role == ROLE_TMA) {
    // ================================================= TMA producer
    // The warp runs the job loop together and each lane issues one box of a
    // job: a single thread issuing TMA one instruction at a time caps at about
    // 20 B/clk per SM, several lanes per instruction do not.
    if (lane == 0) {
      ptx::tma_prefetch_desc(&tm_q);
      ptx::tma_prefetch_desc(&tm_k);
      ptx::tma_prefetch_desc(&tm_v);
    }
    int job = 0;
    bool ok = !p.skip_loads;
    auto wait_all = [&](uint64_t *bar, int parity, int code) {
      const bool got = __all_sync(0xffffffffu, ok && ptx::mbar_wait_backoff(bar, parity, WAIT, 64));
      if (ok && !got) {
        ok = false;
        if (lane == 0) record_err(p, code);
      }
      return ok;
    };
    auto load_kv = [&](bool isv, int q0, int b, int g, int jj) {
      const int slot = job % nslot, use = job / nslot;
      if (use > 0 && !wait_all(bar_free + slot, (use - 1) & 1, ERR_TIMEOUT_FREE)) return;
      const Job jb = job_of(jj, isv);
      const bool last = jb.kt == nkt - 1;
      const CUtensorMap *m = isv ? (last ? &tm_vl : &tm_v) : (last ? &tm_kl : &tm_k);
      const int kb = q0 - p.window + 1;
      if (lane == 0) ptx::mbar_expect_tx(bar_full + slot, jb.ncopy * jb.nh * jb.rows * 256);
      __syncwarp();
      unsigned char *dst = smem + geo.ring_off + slot * TILE_BYTES;
      if (lane < 2 * jb.nh * jb.ncopy) {
        const int c = lane & 1, u = (lane >> 1) % jb.nh, r = (lane >> 1) / jb.nh;
        ptx::tma_load_4d(dst + u * 2 * jb.half + c * jb.half + r * jb.rows * 128, m, bar_full + slot, c * 64,
                         g * HPG + jb.h0 + u, kb + jb.kt * KT_ROWS, b);
      }
      __syncwarp();
      ++job;
    };
    int pq0 = 0, pb = 0, pg = 0;
    int it = 0;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
      int q0, b, g;
      tile_coords(tile, q0, b, g);
      const int buf = it & 1;
      // the Q buffer holds P' of key tile 0 of tile it - 2 until its PV products are complete
      if (it >= 2 && !wait_all(bar_O + buf, ((it - 2) >> 1) & 1, ERR_TIMEOUT_Q)) break;
      if (lane == 0) ptx::mbar_expect_tx(bar_q + buf, NQ * 256);
      __syncwarp();
      if (lane < 2 * HPG) {
        const int h = lane >> 1, c = lane & 1;
        ptx::tma_load_4d(smem + geo.q_off + buf * NQ * 256 + h * BM * 256 + c * BM * 128, &tm_q, bar_q + buf,
                         c * 64, g * HPG + h, q0, b);
      }
      __syncwarp();
      for (int jj = 0; jj < nKk && ok; ++jj) load_kv(false, q0, b, g, jj);
      if (it >= 1)
        for (int jj = 0; jj < nKv && ok; ++jj) load_kv(true, pq0, pb, pg, jj);
      pq0 = q0; pb = b; pg = g;
    }
    if (it >= 1)
      for (int jj = 0; jj < nKv && ok; ++jj) load_kv(true, pq0, pb, pg, jj);
  } else if (role == ROLE_MMA) {
    // ================================================= MMA issuer
    // Whole warp runs the loops; one elected lane issues each tcgen05 op, with
    // descriptors formed as base + offset (cheap to issue back to back).
    const uint32_t ab_fmt = std::is_same<E, __nv_bfloat16>::value ? 1u : 0u;
    const uint32_t idesc_qk = ptx::idesc_f16(ab_fmt, 0, 0, 128, BM);
    const uint32_t idesc_pv = ptx::idesc_f16(ab_fmt, 1, 1, 128, BM);
    const uint32_t ring_addr = ptx::smem_u32(smem + geo.ring_off);
    int job = 0;
    bool ok = true;
    auto wait_u = [&](uint64_t *bar, int parity, int code) {
      const bool got = __all_sync(0xffffffffu, ok && ptx::mbar_wait_backoff(bar, parity, WAIT, 64));
      if (ok && !got) {
        ok = false;
        if (lane == 0) record_err(p, code);
      }
      return ok;
    };
    auto pv = [&](int pit) {
      const int buf = pit & 1;
      if (!wait_u(bar_P + buf, (pit >> 1) & 1, ERR_TIMEOUT_P)) return;
      ptx::tc_fence_after();
      for (int jj = 0; jj < nKv && ok; ++jj, ++job) {
        const int slot = job % nslot;
        if (!wait_u(bar_full + slot, (job / nslot) & 1, ERR_TIMEOUT_FULL)) return;
        ptx::tc_fence_after();
        const Job jb = job_of(jj, true);
        const int nks = jb.rows / 16;
        for (int u = 0; u < jb.nh; ++u) {
          const int h = jb.h0 + u;
          // V: MN-major 128B swizzle, 8-key groups 1024 B apart, d halves jb.half apart
          const uint64_t ad = ptx::smem_desc(ring_addr + slot * TILE_BYTES + u * 2 * jb.half, jb.half, 1024, 2);
          const uint64_t bd =
              ptx::smem_desc(ptx::smem_u32(p_tile(buf, jb.kt)) + h * (jb.rows * BM * 2), BM * 16, 128, 0);
          const uint32_t dd = tbase + buf * 256 + h * BM;
#pragma unroll
          for (int ks = 0; ks < KT_ROWS / 16; ++ks)
            if (ks < nks && ptx::elect_one())
              ptx::mma_f16_ss(dd, ptx::desc_add(ad, ks * 2048), ptx::desc_add(bd, ks * (2 * BM * 16)), idesc_pv,
                              (jb.kt > 0 || ks > 0));
          __syncwarp();
        }
        if (ptx::elect_one()) ptx::mma_commit(bar_free + slot);
        __syncwarp();
      }
      if (ptx::elect_one()) ptx::mma_commit(bar_O + buf);
      __syncwarp();
    };
    int it = 0;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
      const int buf = it & 1;
      // TMEM buffer free once the epilogue of tile it-2 has read its O
      if (it >= 2 && !wait_u(bar_Ofree + buf, ((it - 2) >> 1) & 1, ERR_TIMEOUT_O)) break;
      if (!wait_u(bar_q + buf, (it >> 1) & 1, ERR_TIMEOUT_Q)) break;
      ptx::tc_fence_after();
      const uint64_t qd0 = ptx::smem_desc(ptx::smem_u32(smem + geo.q_off + buf * NQ * 256), 16, 1024, 2);
      for (int jj = 0; jj < nKk && ok; ++jj, ++job) {
        const int slot = job % nslot;
        if (!wait_u(bar_full + slot, (job / nslot) & 1, ERR_TIMEOUT_FULL)) break;
        ptx::tc_fence_after();
        const Job jb = job_of(jj, false);
        for (int u = 0; u < jb.nh; ++u) {
          const int h = jb.h0 + u;
          const uint64_t ad = ptx::smem_desc(
              static_cast<uint32_t>(static_cast<int>(ring_addr + slot * TILE_BYTES + u * 2 * jb.half) + jb.aoff), 16,
              1024, 2);
          const uint64_t bd = ptx::desc_add(qd0, h * BM * 256);
          const uint32_t dd = tbase + buf * 256 + jb.kt * KT_ROWS + h * BM;
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)
            if (ptx::elect_one())
              ptx::mma_f16_ss(dd, ptx::desc_add(ad, (ks >> 2) * jb.half + (ks & 3) * 32),
                              ptx::desc_add(bd, (ks >> 2) * (BM * 128) + (ks & 3) * 32), idesc_qk, ks > 0);
          __syncwarp();
        }
        if (ptx::elect_one()) {
          ptx::mma_commit(bar_free + slot);
          if (jb.h0 + jb.nh == HPG) ptx::mma_commit(bar_S + 2 * buf + jb.kt);
        }
        __syncwarp();
      }
      if (it >= 1 && ok) pv(it - 1);
    }
    if (it >= 1 && ok) pv(it - 1);
  } else if ((role & 0xF0) == ROLE_EPI) {
    // ================================================= epilogue: O^T (lanes = d) -> SMEM -> TMA store
    // 32 columns at a time through an 8 KB staging buffer of its own, so the Q
    // buffer (P' of key tile 0) is free as soon as the PV products are done.
    // Staging layout: [box][d half][RB rows][64 d], one box = RB queries of one head.
    const int quarter = warp & 3, d = 32 * quarter + lane;
    constexpr int RB = BM < 32 ? BM : 32;
    unsigned char *stage = smem + geo.stage_off;
    const bool leader = warp == epi_warp0 && lane == 0;
    int it = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
      int q0, b, g;
      tile_coords(tile, q0, b, g);
      const int buf = it & 1;
      if (!ptx::mbar_wait_backoff(bar_O + buf, (it >> 1) & 1, WAIT, 256)) { record_err(p, ERR_TIMEOUT_O); break; }
      ptx::tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < NQ / 32; ++c) {
        float v[32];
        ptx::tmem_ld<32>(tbase + (static_cast<uint32_t>(32 * quarter) << 16) + buf * 256 + 32 * c, v);
        ptx::tmem_wait_ld();
        if (c == NQ / 32 - 1) {
          // every TMEM read of this tile is done: the buffer may take the next S
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(bar_Ofree + buf);
        }
        ptx::named_bar_sync(2, 128);  // the previous chunk's stores have read the staging buffer
#pragma unroll
        for (int jj = 0; jj < 32; ++jj)
          *reinterpret_cast<E *>(stage + ((jj / RB) * 2 + (d >> 6)) * (RB * 128) + (jj % RB) * 128 + (d & 63) * 2) =
              from_f<E>(v[jj]);
        ptx::fence_proxy_async_smem();
        ptx::named_bar_sync(2, 128);
        if (leader) {
#pragma unroll
          for (int box = 0; box < 32 / RB; ++box) {
            const int col0 = 32 * c + box * RB, h = col0 / BM, i0 = col0 % BM;
#pragma unroll
            for (int dh = 0; dh < 2; ++dh)
              ptx::tma_store_4d(&tm_o, stage + (box * 2 + dh) * (RB * 128), dh * 64, g * HPG + h, q0 + i0, b);
          }
          ptx::bulk_commit();
          ptx::bulk_wait_read0();
        }
      }
    }
    if (leader) ptx::bulk_wait_all0();
  } else if (role != ROLE_IDLE) {
    // ================================================= compose warps
    //
    // For one (query t, key s) pair and one composition set, the HPG heads of
    // the group are mixed as
    //   o[h] = sum_h' M_t[h'][h] a[h'] + kdd_s[h] a[h] + sum_r kw2_s[r][h] sum_h' kw1_s[h'][r] a[h']
    // M_t = w[g] + identity + diag(qdd_t) + qw1_t qw2_t folds every
    // query-dependent term into one HPG x HPG matrix per query, built once per
    // tile; the key-dependent terms come from registers.  The pre set is scaled
    // by scale * log2(e), so composed logits are in base-2 units.
    const int sub = role & 3, kt = role >> 3, cs = (role >> 2) & 1;
    // a warp of the replicated last key tile: its quarter (2 or 3) holds keys
    // 0..31 of the tile, it composes column groups 2 (sub - 2) and the next
    // (one reduction slot, disjoint columns)
    const bool rk = rep_last && kt == nkt - 1;
    const int rw = kt * 4 + (rk ? 0 : sub);
    int cord = 0;  // ordinal of this compose warp among the compose warps
    for (int w = 0; w < warp; ++w) cord += roles.role[w] < 0x40;
    const int ctid = cord * 32 + lane;  // compose-local thread index
    const int g_begin = rk ? 2 * (sub - 2) : cs * (NG / CS), g_end = g_begin + (rk ? 2 : NG / CS);
    const int srow0 = rk ? 0 : 32 * sub;  // first key row of this warp's lanes
    const int s_local = srow0 + lane;
    const int rows_kt = rows_of[kt];
    const float sl2e = p.scale * kLog2e;
    const int G = p.G;
    constexpr int RAWF = HPG * (2 * R + 1);
    constexpr int MF = HPG * HPG;
    constexpr int NM = 2 * BM * MF;      // mixing-matrix entries of one tile (both sets)
    constexpr int MAXREC = 4;            // weight chunks per compose thread (checked by the launcher)
    float *Wt = reinterpret_cast<float *>(smem + geo.wz_off);      // [set][G][h'][h]
    float *raw = reinterpret_cast<float *>(smem + geo.raw_off);    // [set][BM][RAWF]
    float *mrec = reinterpret_cast<float *>(smem + geo.mrec_off);  // [parity][set][BM][h'][h]
    float *redm = reinterpret_cast<float *>(smem + geo.red_off);   // [slot][NQ] column maxima (base 2)
    uint32_t *reds = reinterpret_cast<uint32_t *>(redm + 8 * NQ);  // [slot][NQ] column sums (fixed point)
    float *fac = reinterpret_cast<float *>(smem + geo.fac_off);    // [slot][BM][HPG]
    float kw1[HPG * R], kw2[R * HPG], kdd[HPG];

    // per-query weights of a tile as chunks of HPG contiguous elements: chunk c =
    // (set, query i, k), k = 0: qdd[h]; 1..R: qw1[h][r] (HPG * R contiguous
    // elements cut into R chunks); R+1..2R: qw2[r][h].  Chunk k of a record
    // lands at record floats [k * HPG, (k + 1) * HPG).
    constexpr int NCK = 2 * R + 1;
    constexpr int NCH = 2 * BM * NCK;
    auto chunk_src = [&](int c, int q0, int b, int g) -> const E * {
      const int set = c / (BM * NCK), rem = c % (BM * NCK), i = rem / NCK, k = rem % NCK;
      const TermPtrs &tm = set ? p.post : p.pre;
      const int t = q0 + i, hbase = g * HPG;
      if (t >= T) return nullptr;
      const int64_t tok = (int64_t)b * T + t;
      if (k == 0) return tm.qdd ? elem<E>(tm.qdd, tok * H + hbase) : nullptr;
      if (k <= R) return tm.qw1 ? elem<E>(tm.qw1, (tok * H + hbase) * R + (k - 1) * HPG) : nullptr;
      return tm.qw2 ? elem<E>(tm.qw2, (tok * R + (k - 1 - R)) * H + hbase) : nullptr;
    };
    auto chunk_store = [&](int c, const Raw16<HPG> &v) {
      const int set = c / (BM * NCK), rem = c % (BM * NCK), i = rem / NCK, k = rem % NCK;
      float *dst = raw + (set * BM + i) * RAWF + k * HPG;
#pragma unroll
      for (int h = 0; h < HPG; ++h) dst[h] = raw16_get<E, HPG>(v, h);
    };
    // per-query matrices of a tile (group g) from the raw values -> mrec[par]
    auto build_m = [&](int par, int g, int tid, int nthr) {
      float *dst = mrec + par * NM;
      for (int idx = tid; idx < NM; idx += nthr) {
        const int set = idx / (BM * MF), i = (idx / MF) % BM, h1 = (idx % MF) / HPG, h = idx % HPG;
        const float *rr = raw + (set * BM + i) * RAWF;
        float m = Wt[((set * G + g) * HPG + h1) * HPG + h] + (h1 == h ? rr[h] : 0.f);
#pragma unroll
        for (int r = 0; r < R; ++r) m = fmaf(rr[HPG + h1 * R + r], rr[HPG + HPG * R + r * HPG + h], m);
        // with PAIR the pair layout [set][query / 2][h'][h][query % 2] (compose_m2)
        dst[PAIR ? set * BM * MF + (i >> 1) * 2 * MF + (h1 * HPG + h) * 2 + (i & 1) : idx] = set ? m : m * sl2e;
      }
    };
    // with PAIR the key's weights as duplicated pairs for compose_m2
    ptx::f2_t kw1d[HPG * R], kw2d[R * HPG], kddd[HPG];
    auto load_key = [&](const TermPtrs &tm, float f, int64_t ktok, int hbase, bool key_ok) {
      load_key_weights_vec<E, HPG, R>(tm, ktok, H, hbase, key_ok, kw1, kw2, kdd);
#pragma unroll
      for (int j = 0; j < R * HPG; ++j) kw2[j] *= f;
#pragma unroll
      for (int j = 0; j < HPG; ++j) kdd[j] *= f;
      if constexpr (PAIR) {
#pragma unroll
        for (int j = 0; j < HPG * R; ++j) kw1d[j] = ptx::f2_dup(kw1[j]);
#pragma unroll
        for (int j = 0; j < R * HPG; ++j) kw2d[j] = ptx::f2_dup(kw2[j]);
#pragma unroll
        for (int j = 0; j < HPG; ++j) kddd[j] = ptx::f2_dup(kdd[j]);
      }
    };

    int it = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
      int q0, b, g;
      tile_coords(tile, q0, b, g);
      const int buf = it & 1, hbase = g * HPG;
      const int kb = q0 - p.window + 1;
      const int slen = p.seq_lens ? min(max(p.seq_lens[b], 0), T) : T;
      const int s = kb + kt * KT_ROWS + s_local;
      const bool key_ok = s >= 0 && s < slen && s_local < rows_kt;
      const int wk0 = kb + kt * KT_ROWS + srow0;
      const int khi = min(q0 + BM - 1, slen - 1);
      const bool active = wk0 + 31 >= max(0, kb) && wk0 <= khi && srow0 < rows_kt;
      const int64_t ktok = (int64_t)b * T + s;
      const uint32_t tl = tbase + (static_cast<uint32_t>(32 * sub) << 16) + buf * 256 + kt * KT_ROWS;
      // every (query, key) pair of this warp's keys and the GI queries from t0 is unmasked
      const bool keys_in = wk0 >= 0 && wk0 + 31 < slen && srow0 + 31 < rows_kt;
      auto all_valid = [&](int t0) {
        return keys_in && wk0 + 31 <= t0 && t0 + GI - 1 - wk0 < p.window && t0 + GI - 1 < T;
      };
      auto valid = [&](int t) { return key_ok && s <= t && t - s < p.window && t < T; };
      // issue this tile's key-weight loads first: their latency overlaps the barrier
      if (active) load_key(p.pre, sl2e, ktok, hbase, key_ok);
      if (it == 0) {
        for (int idx = ctid; idx < 2 * G * MF; idx += ncompose) {
          const int set = idx / (G * MF), gg = (idx / MF) % G, h1 = (idx % MF) / HPG, h = idx % HPG;
          const TermPtrs &tm = set ? p.post : p.pre;
          Wt[idx] = (tm.w ? tm.w[((int64_t)gg * HPG + h1) * HPG + h] : 0.f) + (h1 == h && tm.identity ? 1.f : 0.f);
        }
        for (int c = ctid; c < NCH; c += ncompose) {
          const E *src = chunk_src(c, q0, b, g);
          chunk_store(c, src ? ld_raw16<HPG>(src) : raw16_zero<HPG>());
        }
        ptx::named_bar_sync(1, ncompose);
        build_m(0, g, ctid, ncompose);
        if constexpr (EARLY_M) ptx::named_bar_sync(1, ncompose);  // the first tile's matrices are visible
      }
      // (8 heads per group: 64-entry matrices; built after the statistics by all
      // compose threads, and a barrier here makes them visible)
      if constexpr (!EARLY_M) ptx::named_bar_sync(1, ncompose);
      // No barrier between tiles: a tile's matrices are built before the
      // previous tile's second statistics barrier, and a buffer is rewritten
      // only after a barrier that every reader of its last contents has passed
      // (reduction slots: after the combine; factors: after the next tile's
      // first statistics barrier), so warps may run ahead into this tile.
      const float *mcur = mrec + buf * NM;
      bool ok = ptx::mbar_wait(bar_S + 2 * buf + kt, (it >> 1) & 1, WAIT);
      if (!ok) record_err(p, ERR_TIMEOUT_S);
      ptx::tc_fence_after();
      // the next tile's per-query weights: loads issued now, stored after pass 1
      Raw16<HPG> nrv[MAXREC];
      const int ntile = tile + gridDim.x;
      int nq0 = 0, nb = 0, ng = 0;
      if (ntile < ntiles) {
        tile_coords(ntile, nq0, nb, ng);
#pragma unroll
        for (int k = 0; k < MAXREC; ++k) {
          const int c = ctid + k * ncompose;
          const E *src = c < NCH ? chunk_src(c, nq0, nb, ng) : nullptr;
          nrv[k] = src ? ld_raw16<HPG>(src) : raw16_zero<HPG>();
        }
      }

      // ---- pass 1: pre-composition (+ mask at the window's edges), warp-local
      //      column max (redux), e = 2^(S - m_w) back to TMEM, warp-local column
      //      sums.  The sums are exact fixed-point: every e is in [0, 1], and
      //      e + 1 has the value e * 2^23 in its low mantissa bits, so an integer
      //      redux of the bit patterns sums them (minus 32 * bits(1.0), modulo 2^32).
#pragma unroll 1
      for (int grp = g_begin; grp < g_end; ++grp) {
        const int i0 = grp * GI;
        float *mx = redm + rw * NQ + i0;
        uint32_t *sx = reds + rw * NQ + i0;
        if (active && ok) {
          float v[HPG][GI];
#pragma unroll
          for (int h = 0; h < HPG; ++h) ptx::tmem_ld<GI>(tl + h * BM + i0, v[h]);
          ptx::tmem_wait_ld();
          // with PAIR, queries in pairs on .f32x2 (pair base (i0 + ii) * MF in the pair layout)
          if constexpr (!PAIR) {
            const bool full = all_valid(q0 + i0);
#pragma unroll
            for (int ii = 0; ii < GI; ++ii) {
              float a[HPG], o[HPG];
#pragma unroll
              for (int h = 0; h < HPG; ++h) a[h] = v[h][ii];
              compose_m<HPG, R>(a, o, mcur + (i0 + ii) * MF, kw1, kw2, kdd);
              const bool vl = full || valid(q0 + i0 + ii);
#pragma unroll
              for (int h = 0; h < HPG; ++h) v[h][ii] = vl ? o[h] : kMaskedLogit;
            }
          } else if (all_valid(q0 + i0)) {
#pragma unroll
            for (int ii = 0; ii < GI; ii += 2) {
              ptx::f2_t a[HPG], o[HPG];
#pragma unroll
              for (int h = 0; h < HPG; ++h) a[h] = ptx::f2_pack(v[h][ii], v[h][ii + 1]);
              compose_m2<HPG, R>(a, o, mcur + (i0 + ii) * MF, kw1d, kw2d, kddd);
#pragma unroll
              for (int h = 0; h < HPG; ++h) {
                v[h][ii] = ptx::f2_lo(o[h]);
                v[h][ii + 1] = ptx::f2_hi(o[h]);
              }
            }
          } else {
#pragma unroll
            for (int ii = 0; ii < GI; ii += 2) {
              ptx::f2_t a[HPG], o[HPG];
#pragma unroll
              for (int h = 0; h < HPG; ++h) a[h] = ptx::f2_pack(v[h][ii], v[h][ii + 1]);
              compose_m2<HPG, R>(a, o, mcur + (i0 + ii) * MF, kw1d, kw2d, kddd);
              const bool vl0 = valid(q0 + i0 + ii), vl1 = valid(q0 + i0 + ii + 1);
#pragma unroll
              for (int h = 0; h < HPG; ++h) {
                v[h][ii] = vl0 ? ptx::f2_lo(o[h]) : kMaskedLogit;
                v[h][ii + 1] = vl1 ? ptx::f2_hi(o[h]) : kMaskedLogit;
              }
            }
          }
#pragma unroll
          for (int h = 0; h < HPG; ++h) {
            float m8[GI];
            uint32_t s8[GI];
#pragma unroll
            for (int ii = 0; ii < GI; ++ii) {
              m8[ii] = ptx::warp_max(v[h][ii]);
              v[h][ii] = ptx::ex2(v[h][ii] - m8[ii]);
              s8[ii] = ptx::warp_sum_u32(__float_as_uint(v[h][ii] + 1.f));
            }
            if (lane == 0) {
#pragma unroll
              for (int ii = 0; ii < GI; ii += 4) {
                *reinterpret_cast<float4 *>(mx + h * BM + ii) = make_float4(m8[ii], m8[ii + 1], m8[ii + 2], m8[ii + 3]);
                *reinterpret_cast<uint4 *>(sx + h * BM + ii) = make_uint4(s8[ii], s8[ii + 1], s8[ii + 2], s8[ii + 3]);
              }
            }
          }
#pragma unroll
          for (int h = 0; h < HPG; ++h) ptx::tmem_st<GI>(tl + h * BM + i0, v[h]);
        } else if (lane == 0) {
          // nothing of this warp survives the mask: its factor will be 0
#pragma unroll
          for (int h = 0; h < HPG; ++h)
#pragma unroll
            for (int ii = 0; ii < GI; ii += 4) {
              *reinterpret_cast<float4 *>(mx + h * BM + ii) =
                  make_float4(kMaskedLogit, kMaskedLogit, kMaskedLogit, kMaskedLogit);
              *reinterpret_cast<uint4 *>(sx + h * BM + ii) = make_uint4(0u, 0u, 0u, 0u);
            }
        }
      }
      if (ntile < ntiles) {
#pragma unroll
        for (int k = 0; k < MAXREC; ++k) {
          const int c = ctid + k * ncompose;
          if (c < NCH) chunk_store(c, nrv[k]);
        }
      }
      ptx::tmem_wait_st();
      ptx::named_bar_sync(1, ncompose);
      // combine the slots of each column j = h * BM + i: m = max_w m_w,
      // l = sum_w sum_w 2^(m_w - m); factor_w = 2^(m_w - m) / l turns a slot's e
      // into the normalised probability.  A column whose keys are all masked
      // (m at the mask value) gets factor 0: the reference's NaN -> 0 row.
      for (int j = ctid; j < NQ; j += ncompose) {
        float mw[8];
        uint32_t sw[8];
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          mw[w] = w < nslots ? redm[w * NQ + j] : kMaskedLogit;
          sw[w] = w < nslots ? reds[w * NQ + j] : 32u * 0x3F800000u;
        }
        float m = mw[0];
#pragma unroll
        for (int w = 1; w < 8; ++w) m = fmaxf(m, mw[w]);
        float l = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          mw[w] = ptx::ex2(mw[w] - m);
          l = fmaf(mw[w], static_cast<float>(sw[w] - 32u * 0x3F800000u) * 0x1p-23f, l);
        }
        const float il = (m > 0.5f * kMaskedLogit && l > 0.f) ? __frcp_rn(l) : 0.f;
        const int h = j / BM, i = j % BM;
#pragma unroll
        for (int w = 0; w < 8; ++w)
          if (w < nslots)
            fac[w * BM * HPG + (PAIR ? (i >> 1) * 2 * HPG + h * 2 + (i & 1) : i * HPG + h)] = mw[w] * il;
      }
      // the next tile's matrices, from the weights stored after pass 1, built
      // by the compose threads that do not combine columns (all of them when
      // there are no others)
      if constexpr (EARLY_M) {
        const int nb0 = ncompose > NQ ? NQ : 0;
        if (ntile < ntiles && ctid >= nb0) build_m(buf ^ 1, ng, ctid - nb0, ncompose - nb0);
      }
      ptx::named_bar_sync(1, ncompose);
      // post-set key weights into the registers of the pre set (dead after pass 1)
      if (active) load_key(p.post, 1.f, ktok, hbase, key_ok);
      if constexpr (!EARLY_M)
        if (ntile < ntiles) build_m(buf ^ 1, ng, ctid, ncompose);
      // P' of key tile 0 overwrites Q: every QK product of this tile must be complete
      if (ok && kt == 0 && nkt > 1) {
        ok = ptx::mbar_wait(bar_S + 2 * buf + nkt - 1, (it >> 1) & 1, WAIT);
        if (!ok) record_err(p, ERR_TIMEOUT_S);
      }

      // ---- pass 2: normalise, post-composition, P' -> SMEM
      const float *fw = fac + rw * BM * HPG;
      unsigned char *pbase = p_tile(buf, kt) + (s_local & 7) * 16 + (s_local >> 3) * (BM * 16);
#pragma unroll 1
      for (int grp = g_begin; grp < g_end; ++grp) {
        const int i0 = grp * GI;
        float v[HPG][GI];
        if (active && ok) {
#pragma unroll
          for (int h = 0; h < HPG; ++h) ptx::tmem_ld<GI>(tl + h * BM + i0, v[h]);
          ptx::tmem_wait_ld();
          if constexpr (!PAIR) {
#pragma unroll
            for (int ii = 0; ii < GI; ++ii) {
              float a[HPG], o[HPG], f[HPG];
              ld_row<HPG>(fw + (i0 + ii) * HPG, f);
#pragma unroll
              for (int h = 0; h < HPG; ++h) a[h] = v[h][ii] * f[h];
              compose_m<HPG, R>(a, o, mcur + (BM + i0 + ii) * MF, kw1, kw2, kdd);
#pragma unroll
              for (int h = 0; h < HPG; ++h) v[h][ii] = o[h];
            }
          } else
#pragma unroll
          for (int ii = 0; ii < GI; ii += 2) {
            ptx::f2_t a[HPG], o[HPG];
            float f[2 * HPG];
            ld_row<2 * HPG>(fw + (i0 + ii) * HPG, f);  // factors [query / 2][h][query % 2]
#pragma unroll
            for (int h = 0; h < HPG; ++h)
              a[h] = ptx::f2_mul(ptx::f2_pack(v[h][ii], v[h][ii + 1]), ptx::f2_pack(f[2 * h], f[2 * h + 1]));
            compose_m2<HPG, R>(a, o, mcur + (BM + i0 + ii) * MF, kw1d, kw2d, kddd);
#pragma unroll
            for (int h = 0; h < HPG; ++h) {
              v[h][ii] = ptx::f2_lo(o[h]);
              v[h][ii + 1] = ptx::f2_hi(o[h]);
            }
          }
        } else {
#pragma unroll
          for (int h = 0; h < HPG; ++h)
#pragma unroll
            for (int ii = 0; ii < GI; ++ii) v[h][ii] = 0.f;
        }
        if (s_local < rows_kt) {
#pragma unroll
          for (int h = 0; h < HPG; ++h) {
            unsigned char *tile_p = pbase + h * (rows_kt * BM * 2);
#pragma unroll
            for (int c = 0; c < GI; c += 8 < GI ? 8 : GI) {
              // up to 8 queries -> one 16-byte row of an 8x8 core matrix
              constexpr int W8 = GI < 8 ? GI : 8;
              uint32_t pk[W8 / 2];
#pragma unroll
              for (int u = 0; u < W8 / 2; ++u) pk[u] = pack2<E>(v[h][c + 2 * u], v[h][c + 2 * u + 1]);
              const int i = i0 + c;
              unsigned char *dst = tile_p + (i >> 3) * 128 + (i & 7) * 2;
              if constexpr (W8 == 8) {
                *reinterpret_cast<uint4 *>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
              } else if constexpr (W8 == 4) {
                *reinterpret_cast<uint2 *>(dst) = make_uint2(pk[0], pk[1]);
              } else {
                *reinterpret_cast<uint32_t *>(dst) = pk[0];
              }
            }
          }
        }
      }
      ptx::fence_proxy_async_smem();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar_P + buf);
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (role == ROLE_TMA) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tbase, 512);
  }
}

// ------------------------------------------------------------------ host side

template <typename E, int HPG, int R, bool F8 = false>
static cudaError_t launch_t(const dc_attn_params &p, cudaStream_t st) {
  constexpr int BM = NQ / HPG;
  const int nkt = num_key_tiles(HPG, p.window);
  const Geo geo = make_geo(HPG, R, nkt);
  const size_t smem = geo.total + 1024;
  const int rlast = last_tile_rows(HPG, p.window);
  const int64_t sb = (int64_t)p.T * p.H * D, st_ = (int64_t)p.H * D, sh = D;
  CUtensorMap mq, mk, mv, mkl, mvl, mo;
  const bool qk_ok = F8 ? (make_map8(&mq, p.q, p.B, p.T, p.H, BM, sb, st_, sh) &&
                           make_map8(&mk, p.k, p.B, p.T, p.H, KT_ROWS, sb, st_, sh) &&
                           make_map8(&mkl, p.k, p.B, p.T, p.H, rlast, sb, st_, sh))
                        : (make_map(&mq, p.q, p.dtype, p.B, p.T, p.H, BM, sb, st_, sh, true) &&
                           make_map(&mk, p.k, p.dtype, p.B, p.T, p.H, KT_ROWS, sb, st_, sh, true) &&
                           make_map(&mkl, p.k, p.dtype, p.B, p.T, p.H, rlast, sb, st_, sh, true));
  if (!qk_ok ||
      !make_map(&mv, p.v, p.dtype, p.B, p.T, p.H, KT_ROWS, sb, st_, sh, true) ||
      !make_map(&mvl, p.v, p.dtype, p.B, p.T, p.H, rlast, sb, st_, sh, true) ||
      !make_map(&mo, p.out, p.dtype, p.B, p.T, p.H, BM, p.out_sb, p.out_st, p.out_sh, false))
    return cudaErrorInvalidValue;
  TcParams tp;
  tp.B = p.B; tp.T = p.T; tp.H = p.H; tp.G = p.G; tp.window = p.window; tp.slen_default = p.T;
  tp.scale = p.scale;
  tp.seq_lens = p.seq_lens;
  tp.out = p.out;
  tp.out_sb = p.out_sb; tp.out_st = p.out_st; tp.out_sh = p.out_sh;
  tp.err_flag = p.err_flag;
  tp.wait_us = p.wait_us;
  tp.skip_loads = (p.test_flags & DC_TEST_SKIP_LOADS) != 0;
  tp.pre = to_ptrs(p.pre);
  tp.post = to_ptrs(p.post);
  // short windows (<= 2 key tiles): two warps per TMEM lane quarter and key tile
  const int cs = nkt <= 2 ? 2 : 1;
  auto kern = cs == 2 ? dc_tc_kernel<E, HPG, R, 2, 576, F8> : dc_tc_kernel<E, HPG, R, 1, 448, F8>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((p.T + BM - 1) / BM, p.B * p.G);
  dim3 block(32 * (4 * nkt * cs + 2));  // compose warps + TMA warp + MMA warp
  kern<<<grid, block, smem, st>>>(mq, mk, mv, mkl, mvl, mo, tp, nkt, rlast);
  return cudaGetLastError();
}


template <typename E, int HPG, int R>
static cudaError_t launch_p(const dc_attn_params &p, cudaStream_t st) {
  constexpr int BM = NQ / HPG;
  constexpr int CS = 2;
  const int nkt = num_key_tiles(HPG, p.window);
  const int rlast = last_tile_rows(HPG, p.window);
  // deepest K/V ring that fits, at most 3 slots: a 4th slot (SMEM ~226 KB)
  // measured slower, the smaller L1 then serves spills and weight loads worse
  int nslot = 3;
  while (nslot > 2 && make_geo_p(HPG, R, rlast, nslot, p.G).total + 1024 > 227 * 1024) --nslot;
  const size_t smem = make_geo_p(HPG, R, rlast, nslot, p.G).total + 1024;
  // the staged static mixes grow with G: past the shared-memory limit run the per-tile kernel
  if (smem > 227 * 1024) return launch_t<E, HPG, R>(p, st);
  const int64_t sb = (int64_t)p.T * p.H * D, st_ = (int64_t)p.H * D, sh = D;
  CUtensorMap mq, mk, mv, mkl, mvl, mo;
  if (!make_map(&mq, p.q, p.dtype, p.B, p.T, p.H, BM, sb, st_, sh, true) ||
      !make_map(&mk, p.k, p.dtype, p.B, p.T, p.H, KT_ROWS, sb, st_, sh, true) ||
      !make_map(&mv, p.v, p.dtype, p.B, p.T, p.H, KT_ROWS, sb, st_, sh, true) ||
      !make_map(&mkl, p.k, p.dtype, p.B, p.T, p.H, rlast, sb, st_, sh, true) ||
      !make_map(&mvl, p.v, p.dtype, p.B, p.T, p.H, rlast, sb, st_, sh, true) ||
      !make_map(&mo, p.out, p.dtype, p.B, p.T, p.H, BM < 32 ? BM : 32, p.out_sb, p.out_st, p.out_sh, false))
    return cudaErrorInvalidValue;
  TcParams tp;
  tp.B = p.B; tp.T = p.T; tp.H = p.H; tp.G = p.G; tp.window = p.window; tp.slen_default = p.T;
  tp.scale = p.scale;
  tp.seq_lens = p.seq_lens;
  tp.out = p.out;
  tp.out_sb = p.out_sb; tp.out_st = p.out_st; tp.out_sh = p.out_sh;
  tp.err_flag = p.err_flag;
  tp.wait_us = p.wait_us;
  tp.skip_loads = (p.test_flags & DC_TEST_SKIP_LOADS) != 0;
  tp.pre = to_ptrs(p.pre);
  tp.post = to_ptrs(p.post);
  const WarpRoles roles = make_roles(nkt, rlast, CS, HPG);
  // the compose threads prefetch the next tile's per-query records, at most
  // 4 each (MAXREC in the kernel); otherwise run the per-tile kernel
  if (roles.nwarps == 0 || roles.nwarps > 22 || 2 * BM * (2 * R + 1) > 4 * 32 * roles.ncw)
    return launch_t<E, HPG, R>(p, st);
  auto kern = roles.nwarps <= 16   ? dc_tcp_kernel<E, HPG, R, CS, 16>
              : roles.nwarps <= 18 ? dc_tcp_kernel<E, HPG, R, CS, 18>
                                   : dc_tcp_kernel<E, HPG, R, CS, 22>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int ntiles = (p.T + BM - 1) / BM * p.B * p.G;
  dim3 grid(ntiles < sm_count() ? ntiles : sm_count());
  dim3 block(32 * roles.nwarps);
  kern<<<grid, block, smem, st>>>(mq, mk, mv, mkl, mvl, mo, tp, nkt, rlast, nslot, roles);
  return cudaGetLastError();
}

template <typename E, int HPG>
static cudaError_t launch_r(const dc_attn_params &p, cudaStream_t st) {
  // per-query mixing matrices (the decomposed form) run on the one-tile-per-CTA
  // kernel, which folds them into its per-query matrices; the persistent
  // kernel's matrix build stays free of them
  const bool qmat = p.pre.qmat || p.post.qmat;
  if (num_key_tiles(HPG, p.window) <= 2 && !qmat)
    return p.R <= 1 ? launch_p<E, HPG, 1>(p, st) : launch_p<E, HPG, 2>(p, st);
  return p.R <= 1 ? launch_t<E, HPG, 1>(p, st) : launch_t<E, HPG, 2>(p, st);
}

template <typename E>
static cudaError_t launch_e(const dc_attn_params &p, cudaStream_t st) {
  switch (p.H / p.G) {
    case 1: return launch_r<E, 1>(p, st);
    case 2: return launch_r<E, 2>(p, st);
    case 4: return launch_r<E, 4>(p, st);
    case 8: return launch_r<E, 8>(p, st);
  }
  return cudaErrorInvalidValue;
}

template <typename E>
static cudaError_t launch_e8(const dc_attn_params &p, cudaStream_t st) {
  const bool r2 = p.R > 1;
  switch (p.H / p.G) {
    case 1: return r2 ? launch_t<E, 1, 2, true>(p, st) : launch_t<E, 1, 1, true>(p, st);
    case 2: return r2 ? launch_t<E, 2, 2, true>(p, st) : launch_t<E, 2, 1, true>(p, st);
    case 4: return r2 ? launch_t<E, 4, 2, true>(p, st) : launch_t<E, 4, 1, true>(p, st);
    case 8: return r2 ? launch_t<E, 8, 2, true>(p, st) : launch_t<E, 8, 1, true>(p, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace tc

bool tc_supports(const dc_attn_params &p, std::string *why) {
  auto no = [&](const char *m) { if (why) *why = m; return false; };
  const int HPG = p.H / p.G;
  if (p.D != 128) return no("D must be 128");
  if (HPG != 1 && HPG != 2 && HPG != 4 && HPG != 8) return no("heads per group must be 1, 2, 4 or 8");
  if (p.window <= 0) return no("full-causal layers use the SIMT kernel");
  if (tc::num_key_tiles(HPG, p.window) > 3) return no("window too large (BM + window - 1 > 384)");
  if (p.R > 2) return no("rank R > 2");
  if (!(p.scale > 0.f)) return no("non-positive softmax scale");
  auto al = [](const void *x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
  if (!al(p.q) || !al(p.k) || !al(p.v) || !al(p.out)) return no("q, k, v, out must be 16-byte aligned");
  if (p.out_sb % 8 || p.out_st % 8 || p.out_sh % 8) return no("output strides must be multiples of 8 elements");
  return true;
}

// q and k in e4m3 (their scales already folded into p.scale), the rest in p.dtype
cudaError_t launch_tc_fp8qk(const dc_attn_params &p, cudaStream_t st) {
  if (p.dtype == DC_DTYPE_BF16) return tc::launch_e8<__nv_bfloat16>(p, st);
  return tc::launch_e8<__half>(p, st);
}

cudaError_t launch_tc(const dc_attn_params &p, cudaStream_t st) {
  if (p.dtype == DC_DTYPE_BF16) return tc::launch_e<__nv_bfloat16>(p, st);
  return tc::launch_e<__half>(p, st);
}

}  // namespace dcattn
