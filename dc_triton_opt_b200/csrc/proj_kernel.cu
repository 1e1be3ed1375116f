// Producer of the per-token composition weights from the hidden states
// (sm_100a): the step before the DC-attention forward in DCFormer (Xiao et
// al., "Improving Transformers with Dynamically Composable Multi-Head
// Attention", ICML 2024), which the reference project does not contain.
//
//   hidden = gelu(x W1)                                   [M, I]
//   dd     = tanh(x Wdd)  -> pre qdd | pre kdd | post qdd | post kdd   (H each)
//   dw     = hidden W2    -> per set (pre, post): qw1 (H R) | qw2 (R H) | kw1 (H R) | kw2 (R H)
//
// x [W1 | Wdd] with a gelu / tanh epilogue, then hidden W2: on the tensor
// cores through tcgen05 (below) when the shapes fit it (both weight matrices
// of x a multiple of 64 columns, 256 at most together), else through the
// warp-level mma.sync kernel (one launch per weight matrix).  Every output column range of a token is a contiguous run
// in the layout the attention kernels read ([tok][H][R], [tok][R][H],
// [tok][H]), so the epilogue writes each range straight to its tensor: no
// concatenated output and no layout pass.  `hidden` is the only intermediate.
//
// GEMM: C[M, N] = A[M, K] B[K, N], A and B row-major 16-bit, fp32
// accumulation on the tensor cores through warp-level mma.sync m16n8k16;
// 128 x 128 x 32 tiles, 8 warps of 64 x 32, two shared-memory stages filled
// with cp.async.

#include <cuda_runtime.h>

#include <string>
#include <type_traits>

#include "common.cuh"
#include "tc_common.cuh"

namespace dcattn {
namespace proj {

constexpr int TM = 128, TN = 128, TK = 32, NT = 256;
constexpr int AP = TK + 8;   // padded A row (elements)
constexpr int BP = TN + 8;   // padded B row (elements)
constexpr int MAXSEG = 9;

enum Act { ACT_NONE = 0, ACT_GELU = 1, ACT_TANH = 2 };

struct Seg {
  int start, len, act;
  void *dst;  // [M][len], dtype of the call
};

struct GemmParams {
  int M, N, K;
  const void *A, *B;
  const void *B2;  // tensor-core path only: columns [nb, N) come from B2 [K, N - nb]
  int nb;
  int nseg;
  Seg seg[MAXSEG];
};

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

__device__ __forceinline__ uint32_t su32(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void cp16(void *dst, const void *src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(su32(dst)), "l"(src), "r"(ok ? 16 : 0));
}

template <typename E>
__global__ void __launch_bounds__(NT) dc_proj_gemm(const GemmParams p) {
  __shared__ __align__(16) E As[2][TM * AP];
  __shared__ __align__(16) E Bs[2][TK * BP];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm = warp & 1, wn = warp >> 1;  // warp tile 64 x 32 at (wm * 64, wn * 32)
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  const E *A = reinterpret_cast<const E *>(p.A), *B = reinterpret_cast<const E *>(p.B);
  const int nk = p.K / TK;

  auto load = [&](int st, int kt) {
    const int k0 = kt * TK;
    for (int idx = tid; idx < TM * (TK / 8); idx += NT) {  // A: 128 rows x 4 chunks
      const int r = idx / (TK / 8), ch = idx % (TK / 8), m = m0 + r;
      cp16(&As[st][r * AP + ch * 8], A + (int64_t)(m < p.M ? m : 0) * p.K + k0 + ch * 8, m < p.M);
    }
    for (int idx = tid; idx < TK * (TN / 8); idx += NT) {  // B: 32 rows x 16 chunks
      const int r = idx / (TN / 8), ch = idx % (TN / 8), n = n0 + ch * 8;
      cp16(&Bs[st][r * BP + ch * 8], B + (int64_t)(k0 + r) * p.N + (n < p.N ? n : 0), n < p.N);
    }
    asm volatile("cp.async.commit_group;");
  };

  float acc[4][4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;

  load(0, 0);
  for (int kt = 0; kt < nk; ++kt) {
    const int st = kt & 1;
    if (kt + 1 < nk) {
      load(st ^ 1, kt + 1);
      asm volatile("cp.async.wait_group 1;");
    } else {
      asm volatile("cp.async.wait_group 0;");
    }
    __syncthreads();
#pragma unroll
    for (int ks = 0; ks < TK / 16; ++ks) {
      uint32_t af[4][4], bf[4][2];
#pragma unroll
      for (int mi = 0; mi < 4; ++mi) {
        const E *ap = &As[st][(wm * 64 + mi * 16 + (lane & 15)) * AP + ks * 16 + (lane >> 4) * 8];
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(af[mi][0]), "=r"(af[mi][1]), "=r"(af[mi][2]), "=r"(af[mi][3]) : "r"(su32(ap)));
      }
#pragma unroll
      for (int ni = 0; ni < 4; ++ni) {
        const E *bp = &Bs[st][(ks * 16 + (lane & 15)) * BP + wn * 32 + ni * 8];
        asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
                     : "=r"(bf[ni][0]), "=r"(bf[ni][1]) : "r"(su32(bp)));
      }
#pragma unroll
      for (int mi = 0; mi < 4; ++mi)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni) mma16816<E>(acc[mi][ni], af[mi], bf[ni]);
    }
    __syncthreads();
  }

  // epilogue: route each column to its segment (tensor), apply the activation
  const int g8 = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int ni = 0; ni < 4; ++ni)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int n = n0 + wn * 32 + ni * 8 + 2 * t4 + e;
      if (n >= p.N) continue;
      int si = 0;
      while (si + 1 < p.nseg && n >= p.seg[si + 1].start) ++si;
      const Seg &sg = p.seg[si];
      E *dst = reinterpret_cast<E *>(sg.dst);
#pragma unroll
      for (int mi = 0; mi < 4; ++mi)
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int m = m0 + wm * 64 + mi * 16 + g8 + half * 8;
          if (m >= p.M) continue;
          float v = acc[mi][ni][half * 2 + e];
          if (sg.act == ACT_GELU) v = 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
          else if (sg.act == ACT_TANH) v = tanhf(v);
          dst[(int64_t)m * sg.len + (n - sg.start)] = from_f<E>(v);
        }
    }
}

template <typename E>
static cudaError_t launch(const GemmParams &p, cudaStream_t st) {
  dim3 grid((p.N + TN - 1) / TN, (p.M + TM - 1) / TM);
  dc_proj_gemm<E><<<grid, NT, 0, st>>>(p);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- tcgen05 GEMM
// C[M, N] = A[M, K] [B1 | B2][K, N] for N <= 256: one CTA owns 128 rows and
// every column, so x is read once for both weight matrices.  TMA loads A as
// 128 x 64 K-major tiles and each B as 64 x 64 MN-major tiles (both 128-byte
// swizzled) into a 4-stage ring; one thread issues M = 128, N = N MMAs into a
// TMEM accumulator; four warps (one per TMEM lane quarter) apply the
// activation, stage the tile in shared memory and write every segment with
// coalesced 16-byte stores.  Every wait is bounded; a wait that runs out writes
// a code to `err` and the CTA skips the rest of its work.
constexpr int TC_STAGES = 4, TC_KC = 64, TC_ABYTES = 128 * TC_KC * 2, TC_BCHUNK = TC_KC * 64 * 2;
constexpr int TC_SROW = 256 + 8;  // staging row (elements)

struct TcGemm {
  int M, N, K, nb;  // columns [0, nb) from B1, [nb, N) from B2
  int nseg;
  Seg seg[MAXSEG];
  int32_t *err;
  uint32_t wait_us;
  int stages;      // ring depth (<= TC_STAGES; short K loops need fewer)
  int ring_bytes;  // max(stages * stage bytes, epilogue staging)
};

template <typename E>
__global__ void __launch_bounds__(192, 1)
    dc_proj_tc_gemm(const __grid_constant__ CUtensorMap ma, const __grid_constant__ CUtensorMap mb1,
                    const __grid_constant__ CUtensorMap mb2, const TcGemm p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                          ~static_cast<uintptr_t>(1023));
  const int nbc = p.N / 64;                           // 64-column B chunks
  const int stage_bytes = TC_ABYTES + nbc * TC_BCHUNK;
  const int NS = p.stages;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + p.ring_bytes);
  uint64_t *full = bars, *freeb = bars + NS, *done = bars + 2 * NS;
  uint32_t *tslot = reinterpret_cast<uint32_t *>(done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * 128, nk = p.K / TC_KC;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      ptx::mbar_init(full + i, 1);
      ptx::mbar_init(freeb + i, 1);
    }
    ptx::mbar_init(done, 1);
    ptx::fence_mbar_init();
  }
  if (warp == 1) ptx::tmem_alloc(tslot, 256);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tbase = *tslot;
  auto fail = [&](int code) { atomicCAS(p.err, 0, code); };

  if (warp == 0) {
    // one thread's TMA loads are processed one after another, so the loads of
    // a stage go out from several lanes: lane 0 the A tile, lane 1 + c B chunk c
    for (int kt = 0; kt < nk; ++kt) {
      const int st = kt % NS, use = kt / NS;
      bool ok = true;
      if (lane == 0 && use > 0) ok = ptx::mbar_wait(freeb + st, (use - 1) & 1, p.wait_us);
      if (!__shfl_sync(0xffffffffu, ok, 0)) {
        if (lane == 0) fail(tc::ERR_TIMEOUT_FREE);
        break;
      }
      unsigned char *dst = smem + st * stage_bytes;
      if (lane == 0) ptx::mbar_expect_tx(full + st, stage_bytes);
      __syncwarp();
      if (lane == 0) {
        ptx::tma_load_2d(dst, &ma, full + st, kt * TC_KC, m0);
      } else if (lane <= nbc) {
        const int c = lane - 1;
        const bool first = c * 64 < p.nb;
        ptx::tma_load_2d(dst + TC_ABYTES + c * TC_BCHUNK, first ? &mb1 : &mb2, full + st,
                         first ? c * 64 : c * 64 - p.nb, kt * TC_KC);
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    const uint32_t ab = std::is_same<E, __nv_bfloat16>::value ? 1u : 0u;
    const uint32_t idesc = ptx::idesc_f16(ab, 0, 1, 128, p.N);
    const uint64_t ad0 = ptx::smem_desc(ptx::smem_u32(smem), 16, 1024, 2);
    const uint64_t bd0 = ptx::smem_desc(ptx::smem_u32(smem + TC_ABYTES), TC_BCHUNK, 1024, 2);
    bool ok = true;
    for (int kt = 0; kt < nk && ok; ++kt) {
      const int st = kt % NS;
      ok = __all_sync(0xffffffffu, ptx::mbar_wait(full + st, (kt / NS) & 1, p.wait_us));
      if (!ok) {
        if (lane == 0) fail(tc::ERR_TIMEOUT_FULL);
        break;
      }
      ptx::tc_fence_after();
      const uint64_t ad = ptx::desc_add(ad0, st * stage_bytes), bd = ptx::desc_add(bd0, st * stage_bytes);
#pragma unroll
      for (int ks = 0; ks < TC_KC / 16; ++ks)
        if (ptx::elect_one())
          ptx::mma_f16_ss(tbase, ptx::desc_add(ad, ks * 32), ptx::desc_add(bd, ks * 2048), idesc, kt > 0 || ks > 0);
      if (ptx::elect_one()) ptx::mma_commit(freeb + st);
      __syncwarp();
    }
    if (ok && ptx::elect_one()) ptx::mma_commit(done);
    __syncwarp();
  } else {
    // ---- epilogue: warps 2..5, lane quarter warp % 4 holds rows 32 q .. 32 q + 31
    const int q = warp & 3, r = 32 * q + lane;
    E *stage = reinterpret_cast<E *>(smem);  // the ring is idle once every MMA is done
    const bool ok = ptx::mbar_wait(done, 0, p.wait_us);
    if (!ok && lane == 0) fail(tc::ERR_TIMEOUT_O);
    ptx::tc_fence_after();
    if (__all_sync(0xffffffffu, ok)) {
      for (int c0 = 0; c0 < p.N; c0 += 32) {
        float v[32];
        ptx::tmem_ld<32>(tbase + (static_cast<uint32_t>(32 * q) << 16) + c0, v);
        ptx::tmem_wait_ld();
        int si = 0;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int n = c0 + j;
          while (si + 1 < p.nseg && n >= p.seg[si + 1].start) ++si;
          float x = v[j];
          if (p.seg[si].act == ACT_GELU) x = 0.5f * x * (1.f + erff(x * 0.70710678118654752f));
          else if (p.seg[si].act == ACT_TANH) x = tanhf(x);
          stage[r * TC_SROW + n] = from_f<E>(x);
        }
      }
    }
    ptx::named_bar_sync(1, 128);
    if (ok) {
      const int rows = min(128, p.M - m0), tid = threadIdx.x - 64;
      for (int si = 0; si < p.nseg; ++si) {
        const Seg &sg = p.seg[si];
        E *dst = reinterpret_cast<E *>(sg.dst) + (int64_t)m0 * sg.len;
        if (sg.len % 8 == 0) {
          const int cpr = sg.len / 8;  // 16-byte chunks per row
          for (int idx = tid; idx < rows * cpr; idx += 128) {
            const int rr = idx / cpr, ch = idx % cpr;
            *reinterpret_cast<uint4 *>(dst + (int64_t)rr * sg.len + ch * 8) =
                *reinterpret_cast<const uint4 *>(stage + rr * TC_SROW + sg.start + ch * 8);
          }
        } else {
          for (int idx = tid; idx < rows * sg.len; idx += 128)
            dst[idx] = stage[(idx / sg.len) * TC_SROW + sg.start + idx % sg.len];
        }
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tbase, 256);
  }
}

// 2-D map of a row-major [rows, cols] 16-bit matrix, box {64 cols, box_rows}, 128-byte swizzle
static bool map2d(CUtensorMap *m, const void *base, int dtype, int rows, int cols, int box_rows) {
  tc::EncodeTiledFn enc = tc::get_encode();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt =
      dtype == DC_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return enc(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// the tensor-core GEMM runs when both B matrices have a multiple of 64 columns,
// N <= 256 and K is a multiple of 64
static bool tc_fits(int K, int n1, int n2) {
  return K % TC_KC == 0 && n1 % 64 == 0 && n2 % 64 == 0 && n1 + n2 <= 256 && n1 + n2 >= 64;
}

}  // namespace proj

// The tcgen05 path for x [W1 | Wdd] and hidden W2 when their shapes fit it,
// the mma.sync kernel otherwise.
template <typename E>
static cudaError_t launch_one(const proj::GemmParams &g, int dtype, int32_t *err, cudaStream_t st) {
  using namespace proj;
  const int n1 = g.B2 ? g.nb : g.N, n2 = g.N - n1;
  if (!tc_fits(g.K, n1, n2)) return launch<E>(g, st);
  CUtensorMap ma, mb1, mb2;
  if (!map2d(&ma, g.A, dtype, g.M, g.K, 128) || !map2d(&mb1, g.B, dtype, g.K, n1, TC_KC) ||
      !map2d(&mb2, g.B2 ? g.B2 : g.B, dtype, g.K, g.B2 ? n2 : n1, TC_KC))
    return cudaErrorInvalidValue;
  TcGemm t{};
  t.M = g.M; t.N = g.N; t.K = g.K; t.nb = n1; t.nseg = g.nseg;
  for (int i = 0; i < g.nseg; ++i) t.seg[i] = g.seg[i];
  t.err = err;
  t.wait_us = 2000000u;
  // a ring no deeper than the K loop: a short one (hidden W2, K = 128) then
  // fits two CTAs per SM
  t.stages = g.K / TC_KC < TC_STAGES ? g.K / TC_KC : TC_STAGES;
  const int sb = TC_ABYTES + (g.N / 64) * TC_BCHUNK, staging = 128 * TC_SROW * 2;
  t.ring_bytes = t.stages * sb > staging ? t.stages * sb : (staging + 1023) / 1024 * 1024;
  const int smem = t.ring_bytes + 8 * (2 * t.stages + 2) + 1024;
  auto kern = dc_proj_tc_gemm<E>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kern<<<(g.M + 127) / 128, 192, smem, st>>>(ma, mb1, mb2, t);
  return cudaGetLastError();
}

cudaError_t launch_proj(const dc_proj_params &q, void *hidden, int32_t *err, cudaStream_t st) {
  using namespace proj;
  const int H = q.H, HR = q.H * q.R;
  GemmParams g1{};  // x [W1 | Wdd]: gelu -> hidden, tanh -> the four gates
  g1.M = q.M; g1.N = q.I + 4 * H; g1.K = q.Dm; g1.A = q.x; g1.B = q.w1; g1.B2 = q.wdd; g1.nb = q.I;
  g1.nseg = 5;
  g1.seg[0] = {0, q.I, ACT_GELU, hidden};
  for (int i = 0; i < 4; ++i) g1.seg[1 + i] = {q.I + i * H, H, ACT_TANH, q.dd[i]};
  GemmParams g2{};  // hidden W2 -> the eight rank-R weight tensors
  g2.M = q.M; g2.N = 8 * HR; g2.K = q.I; g2.A = hidden; g2.B = q.w2; g2.nb = g2.N;
  g2.nseg = 8;
  for (int i = 0; i < 8; ++i) g2.seg[i] = {i * HR, HR, ACT_NONE, q.dw[i]};
  const bool bf = q.dtype == DC_DTYPE_BF16;
  const bool fused = tc_fits(q.Dm, q.I, 4 * H);
  cudaError_t e;
  if (fused) {
    e = bf ? launch_one<__nv_bfloat16>(g1, q.dtype, err, st) : launch_one<__half>(g1, q.dtype, err, st);
  } else {  // the mma.sync kernel reads one B matrix: two launches over x
    GemmParams ga = g1, gd = g1;
    ga.N = q.I; ga.B2 = nullptr; ga.nb = q.I; ga.nseg = 1;
    gd.N = 4 * H; gd.B = q.wdd; gd.B2 = nullptr; gd.nb = 4 * H; gd.nseg = 4;
    for (int i = 0; i < 4; ++i) gd.seg[i] = {i * H, H, ACT_TANH, q.dd[i]};
    e = bf ? launch<__nv_bfloat16>(ga, st) : launch<__half>(ga, st);
    if (e == cudaSuccess) e = bf ? launch<__nv_bfloat16>(gd, st) : launch<__half>(gd, st);
  }
  if (e != cudaSuccess) return e;
  return bf ? launch_one<__nv_bfloat16>(g2, q.dtype, err, st) : launch_one<__half>(g2, q.dtype, err, st);
}

}  // namespace dcattn
