// Producer of the per-token composition weights from the hidden states
// (sm_100a): the step before the DC-attention forward in DCFormer (Xiao et
// al., "Improving Transformers with Dynamically Composable Multi-Head
// Attention", ICML 2024), which the reference project does not contain.
//
//   hidden = gelu(x W1)                                   [M, I]
//   dd     = tanh(x Wdd)  -> pre qdd | pre kdd | post qdd | post kdd   (H each)
//   dw     = hidden W2    -> per set (pre, post): qw1 (H R) | qw2 (R H) | kw1 (H R) | kw2 (R H)
//
// Two launches of one GEMM kernel (x [W1 | Wdd] with a gelu / tanh epilogue,
// then hidden W2).  Every output column range of a token is a contiguous run
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

}  // namespace proj

cudaError_t launch_proj(const dc_proj_params &q, void *hidden, cudaStream_t st) {
  using namespace proj;
  const int H = q.H, R = q.R, HR = q.H * q.R;
  // x [W1 | Wdd]: W1 and Wdd are two row-major [Dm, *] matrices, so the first
  // GEMM runs twice over x (once per matrix); both reads of x come from L2 for
  // any practical M tile order.
  GemmParams g1{};
  g1.M = q.M; g1.N = q.I; g1.K = q.Dm; g1.A = q.x; g1.B = q.w1;
  g1.nseg = 1;
  g1.seg[0] = {0, q.I, ACT_GELU, hidden};
  GemmParams gd{};
  gd.M = q.M; gd.N = 4 * H; gd.K = q.Dm; gd.A = q.x; gd.B = q.wdd;
  gd.nseg = 4;
  for (int i = 0; i < 4; ++i) gd.seg[i] = {i * H, H, ACT_TANH, q.dd[i]};
  GemmParams g2{};
  g2.M = q.M; g2.N = 8 * HR; g2.K = q.I; g2.A = hidden; g2.B = q.w2;
  g2.nseg = 8;
  for (int i = 0; i < 8; ++i) g2.seg[i] = {i * HR, HR, ACT_NONE, q.dw[i]};
  (void)R;
  cudaError_t e;
  const bool bf = q.dtype == DC_DTYPE_BF16;
  for (const GemmParams *g : {&g1, &gd, &g2}) {
    e = bf ? proj::launch<__nv_bfloat16>(*g, st) : proj::launch<__half>(*g, st);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace dcattn
