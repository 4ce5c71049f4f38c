// gates.cu -- chunk-local cumulative gate, the upstream producer of g.
//
//   g[b, c*BT + i, h] = scale * sum_{j <= i} g_inc[b, c*BT + j, h]
//
// for every BT = 64-token chunk c, summed in order in fp32. The reference's
// generators build g exactly this way from per-token increments
// (kernels/chunk_fwd_h/reference.py:41-45, kernels/recompute_w_u/reference.py:
// 103-106); every DeltaNet op of this library takes g in that form.
//
// One thread per (b, chunk, h): its 64 loads are issued together (a warp reads
// 32 consecutive heads, i.e. contiguous bytes of a row), then summed in order.
// Each thread reads only the elements it writes, so g_out may alias g_inc.
#include "host_util.h"

namespace thm {
namespace gates {

constexpr int kBT = 64;

__global__ void __launch_bounds__(256) chunk_local_cumsum_kernel(const float* in, float* out, long long ncols,
                                                                 int H, float scale) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // (b, chunk, h)
  if (i >= ncols) return;
  const long long bc = i / H;
  const int h = (int)(i - bc * H);
  const long long base = bc * kBT * H + h;  // row (b*T + c*BT), head h
  float v[kBT];
#pragma unroll
  for (int r = 0; r < kBT; ++r) v[r] = in[base + (long long)r * H];
  float acc = 0.f;
#pragma unroll
  for (int r = 0; r < kBT; ++r) {
    acc += v[r];
    out[base + (long long)r * H] = acc * scale;
  }
}

}  // namespace gates
}  // namespace thm

extern "C" int thm_chunk_local_cumsum_fwd(const float* g_inc, float* g, int B, int T, int H, float scale,
                                          thm_stream_t stream) {
  using namespace thm;
  if (B < 0 || T < 0 || H < 0 || T % 64 != 0) return THM_ERR_INVALID;
  if ((long long)B * T * H == 0) return THM_OK;
  if (!g_inc || !g) return THM_ERR_INVALID;
  const long long ncols = (long long)B * (T / 64) * H;
  const long long blocks = (ncols + 255) / 256;
  if (blocks > 0x7fffffffLL) return THM_ERR_UNSUPPORTED;
  gates::chunk_local_cumsum_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      g_inc, g, ncols, H, scale);
  return check_launch();
}
