// sp_fold.cu -- prefix fold of per-segment affine state maps (sequence parallel).
//
// The delta-rule state recurrence of a segment of chunks is affine in the state
// entering it (kernels/chunk_fwd_h/kernel.py:61-138 extended with the delta
// rule): h_out = M h_in + S, with M [K, K] and S [K, V] per (batch, head). Given
// the maps of R consecutive segments, the states entering them are
//
//   x_0 = h0 (or 0),   x_{r+1} = M_r x_r + S_r,
//
// and x_R is the state after the last one. One launch computes x_0 .. x_{nout-1}
// for every (b, h): one CTA per (b, h, 32-column tile of V) keeps its K x 32
// tile of x in shared memory across the R steps; a thread owns 4 rows x 4
// columns and reads its rows of M as float4 (fp32 throughout). The same kernel
// composes maps: with x_0 = [I | 0] and S_r = [0 | S_r] over K + V columns it
// yields [prod M | composed S].
#include "host_util.h"

namespace thm {
namespace spfold {

constexpr int kThreads = 256;
constexpr int kCols = 32;   // columns of x per CTA
constexpr int kMaxK = 128;  // 32 row groups of 4 x 8 column groups of 4

__global__ void __launch_bounds__(kThreads) sp_fold_kernel(const float* __restrict__ M, const float* __restrict__ S,
                                                           const float* __restrict__ x0, float* __restrict__ out,
                                                           int nout, int BH, int K, int V) {
  __shared__ __align__(16) float X[kMaxK][kCols + 4];
  const int tid = threadIdx.x;
  const long long bh = blockIdx.y;
  const int v0 = blockIdx.x * kCols;
  const int i0 = 4 * (tid >> 3), j0 = 4 * (tid & 7);
  const bool active = i0 < K;

  // x_0
  for (int idx = tid; idx < K * kCols; idx += kThreads) {
    const int r = idx / kCols, c = idx - r * kCols;
    const long long o = (bh * K + r) * V + v0 + c;
    const float v = x0 != nullptr ? x0[o] : 0.f;
    X[r][c] = v;
    out[o] = v;
  }
  __syncthreads();
  for (int s = 0; s + 1 < nout; ++s) {
    const float* Ms = M + ((long long)s * BH + bh) * K * K;
    const float* Ss = S + ((long long)s * BH + bh) * K * V + v0 + j0;
    float acc[4][4];
    if (active) {
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const float4 sv = *reinterpret_cast<const float4*>(Ss + (long long)(i0 + a) * V);
        acc[a][0] = sv.x; acc[a][1] = sv.y; acc[a][2] = sv.z; acc[a][3] = sv.w;
      }
      for (int k = 0; k < K; k += 4) {
        float4 m[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) m[a] = __ldg(reinterpret_cast<const float4*>(Ms + (long long)(i0 + a) * K + k));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const float4 x = *reinterpret_cast<const float4*>(&X[k + kk][j0]);
#pragma unroll
          for (int a = 0; a < 4; ++a) {
            const float mv = kk == 0 ? m[a].x : kk == 1 ? m[a].y : kk == 2 ? m[a].z : m[a].w;
            acc[a][0] = fmaf(mv, x.x, acc[a][0]);
            acc[a][1] = fmaf(mv, x.y, acc[a][1]);
            acc[a][2] = fmaf(mv, x.z, acc[a][2]);
            acc[a][3] = fmaf(mv, x.w, acc[a][3]);
          }
        }
      }
    }
    __syncthreads();  // every thread has read x_s
    if (active) {
      float* o = out + (((long long)(s + 1) * BH + bh) * K + i0) * V + v0 + j0;
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const float4 r4 = make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
        *reinterpret_cast<float4*>(&X[i0 + a][j0]) = r4;
        *reinterpret_cast<float4*>(o + (long long)a * V) = r4;
      }
    }
    __syncthreads();
  }
}

}  // namespace spfold
}  // namespace thm

extern "C" int thm_sp_prefix_fold(const float* M, const float* S, const float* x0, float* out, int nout, int BH,
                                  int K, int V, thm_stream_t stream) {
  using namespace thm;
  if (nout < 1 || BH < 0 || K <= 0 || V <= 0) return THM_ERR_INVALID;
  if (BH == 0) return THM_OK;
  if (!out || (nout > 1 && (!M || !S))) return THM_ERR_INVALID;
  if (K > spfold::kMaxK || K % 4 != 0 || V % spfold::kCols != 0) return THM_ERR_UNSUPPORTED;
  if (!aligned16(out) || (M && !aligned16(M)) || (S && !aligned16(S)) || (x0 && !aligned16(x0)))
    return THM_ERR_ALIGNMENT;
  if (BH > 65535) return THM_ERR_UNSUPPORTED;
  dim3 grid(V / spfold::kCols, BH);
  spfold::sp_fold_kernel<<<grid, spfold::kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(M, S, x0, out, nout,
                                                                                               BH, K, V);
  return check_launch();
}
