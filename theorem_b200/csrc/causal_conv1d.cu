// causal_conv1d.cu -- depthwise causal 1-D convolution (Mamba-2 style).
//
// Replaces the reference's Triton kernel (kernels/causal_conv1d/kernel.py:44-117)
// and its launcher (:170-230). Pure HBM streaming: every input element is
// read from DRAM once and every output written once; the W-1 halo is re-read
// from L1 (BDS) or carried in registers (BSD).
//
//   out[b,d,t] = act(bias[d] + sum_{k<W} weight[d,k] * x[b,d,t-W+1+k])
//
// BDS ([B,D,S], S contiguous, fp32): copy-shaped float4 access (each warp
//   instruction covers 512 contiguous bytes of a row); the halo comes from
//   the neighbouring lane by warp shuffle (lane 0 reads it from memory).
// BSD ([B,S,D], D contiguous, fp32/bf16): one thread = 4 consecutive channels
//   x a 256-step time strip, software-pipelined in tiles of 8 rows; 8-byte
//   (bf16) or 16-byte (fp32) loads (a warp covers 128 consecutive channels),
//   the W-1 previous rows held in registers; optional SiLU and per-group L2
//   norm (warp shuffles over G/4 lanes) fused into the store.
#include <cuda_bf16.h>

#include "host_util.h"
#include "sm100.cuh"

THM_DEFINE_STATUS(g_status_conv)

namespace thm {
namespace conv {

// x * sigmoid(x) with the fast exp / divide intrinsics (rel. error ~1e-6; the
// quotient goes to 0 for x < -88 where exp(-x) overflows).
__device__ __forceinline__ float silu_f(float v) { return __fdividef(v, 1.0f + __expf(-v)); }

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// ---------------------------------------------------------------------------
// BDS, fp32, S % 4 == 0, W <= 5: copy-shaped access. CTA (row, chunk) of a
// [B*D, S] view; each warp owns 64 consecutive float4 of one row and thread
// `lane` takes float4 base + 32 j + lane (j = 0, 1), so every load and store
// instruction of a warp covers 512 contiguous bytes. The W-1 <= 4 inputs
// before a float4 are the previous float4: lane-1's (shuffle), lane 31's of
// the previous j, or (lane 0, j = 0) one extra load; zeros at the row start.
// d and the W weights are uniform per CTA.
// ---------------------------------------------------------------------------
constexpr int kBdsThreads = 128;
constexpr int kBdsNJ = 2;
constexpr int kBdsQ = kBdsThreads * kBdsNJ;  // float4 per CTA

template <int W, bool SILU>
__global__ void __launch_bounds__(kBdsThreads) conv_bds_f4(const float* __restrict__ x, const float* __restrict__ w,
                                                          const float* __restrict__ bias, float* __restrict__ out,
                                                          int D, int S) {
  static_assert(W >= 1 && W <= 5, "one previous float4 holds the halo");
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int row = blockIdx.x;
  const int d = row % D;
  const int nq = S >> 2;
  const int base = blockIdx.y * kBdsQ + wid * (32 * kBdsNJ);
  const float4* xr = reinterpret_cast<const float4*>(x + (long long)row * S);
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 c[kBdsNJ];
#pragma unroll
  for (int j = 0; j < kBdsNJ; ++j) {
    const int q = base + 32 * j + lane;
    c[j] = q < nq ? __ldg(xr + q) : z4;
  }
  const float4 pm = (lane == 0 && base > 0 && base <= nq) ? __ldg(xr + base - 1) : z4;
  float wk[W];
#pragma unroll
  for (int k = 0; k < W; ++k) wk[k] = __ldg(w + (long long)d * W + k);
  const float bd = __ldg(bias + d);
  float4* orow = reinterpret_cast<float4*>(out + (long long)row * S);
#pragma unroll
  for (int j = 0; j < kBdsNJ; ++j) {
    float4 p = make_float4(__shfl_up_sync(0xffffffffu, c[j].x, 1), __shfl_up_sync(0xffffffffu, c[j].y, 1),
                           __shfl_up_sync(0xffffffffu, c[j].z, 1), __shfl_up_sync(0xffffffffu, c[j].w, 1));
    if (j > 0) {
      const float4& cp = c[j > 0 ? j - 1 : 0];
      const float4 l31 = make_float4(__shfl_sync(0xffffffffu, cp.x, 31), __shfl_sync(0xffffffffu, cp.y, 31),
                                     __shfl_sync(0xffffffffu, cp.z, 31), __shfl_sync(0xffffffffu, cp.w, 31));
      if (lane == 0) p = l31;
    } else if (lane == 0) {
      p = pm;
    }
    const int q = base + 32 * j + lane;
    if (q >= nq) continue;
    const float v[8] = {p.x, p.y, p.z, p.w, c[j].x, c[j].y, c[j].z, c[j].w};
    float o[4];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      float acc = bd;
#pragma unroll
      for (int k = 0; k < W; ++k) acc = fmaf(v[4 + jj - (W - 1) + k], wk[k], acc);
      o[jj] = SILU ? silu_f(acc) : acc;
    }
    orow[q] = make_float4(o[0], o[1], o[2], o[3]);
  }
}

// ---------------------------------------------------------------------------
// BDS, fp32, S % 4 == 0, 6 <= W <= 8: one thread = 8 consecutive outputs of a
// row, float4 loads/stores; the halo comes from the neighbouring lane by warp
// shuffle (lane 0 reads it from memory).
// ---------------------------------------------------------------------------
template <int W, bool SILU>
__global__ void __launch_bounds__(256) conv_bds_vec8(const float* __restrict__ x, const float* __restrict__ w,
                                                     const float* __restrict__ bias, float* __restrict__ out,
                                                     int D, int S, long long nseg_total, int nseg_row) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int lane = threadIdx.x & 31;
  const bool valid = i < nseg_total;
  const long long ii = valid ? i : nseg_total - 1;
  const long long row = ii / nseg_row;
  const int seg = (int)(ii - row * nseg_row);
  const int d = (int)(row % D);
  const int t0 = seg * 8;
  const float* xr = x + row * (long long)S;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);

  const bool has_hi = (t0 + 4) < S;
  float4 c0 = ldg4(xr + t0);
  float4 c1 = has_hi ? ldg4(xr + t0 + 4) : z4;
  float pv[8] = {__shfl_up_sync(0xffffffffu, c0.x, 1), __shfl_up_sync(0xffffffffu, c0.y, 1),
                 __shfl_up_sync(0xffffffffu, c0.z, 1), __shfl_up_sync(0xffffffffu, c0.w, 1),
                 __shfl_up_sync(0xffffffffu, c1.x, 1), __shfl_up_sync(0xffffffffu, c1.y, 1),
                 __shfl_up_sync(0xffffffffu, c1.z, 1), __shfl_up_sync(0xffffffffu, c1.w, 1)};
  if (seg == 0) {
#pragma unroll
    for (int j = 0; j < 8; ++j) pv[j] = 0.f;
  } else if (lane == 0) {
    const float4 p2 = (W > 5) ? ldg4(xr + t0 - 8) : z4;
    const float4 p1 = ldg4(xr + t0 - 4);
    pv[0] = p2.x; pv[1] = p2.y; pv[2] = p2.z; pv[3] = p2.w;
    pv[4] = p1.x; pv[5] = p1.y; pv[6] = p1.z; pv[7] = p1.w;
  }
  if (!valid) return;

  float v[16] = {pv[0], pv[1], pv[2], pv[3], pv[4], pv[5], pv[6], pv[7],
                 c0.x,  c0.y,  c0.z,  c0.w,  c1.x,  c1.y,  c1.z,  c1.w};
  float wk[W];
#pragma unroll
  for (int k = 0; k < W; ++k) wk[k] = __ldg(w + (long long)d * W + k);
  const float bd = __ldg(bias + d);

  float o[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float acc = bd;
#pragma unroll
    for (int k = 0; k < W; ++k) acc = fmaf(v[8 + j - (W - 1) + k], wk[k], acc);
    o[j] = SILU ? silu_f(acc) : acc;
  }
  float* orow = out + row * (long long)S + t0;
  *reinterpret_cast<float4*>(orow) = make_float4(o[0], o[1], o[2], o[3]);
  if (has_hi) *reinterpret_cast<float4*>(orow + 4) = make_float4(o[4], o[5], o[6], o[7]);
}

// ---------------------------------------------------------------------------
// BDS, fp32, any S / W / alignment: one output per thread.
// ---------------------------------------------------------------------------
template <bool SILU>
__global__ void __launch_bounds__(256) conv_bds_scalar(const float* __restrict__ x, const float* __restrict__ w,
                                                       const float* __restrict__ bias, float* __restrict__ out,
                                                       int D, int S, int W, long long total) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const long long row = i / S;
  const int t = (int)(i - row * S);
  const int d = (int)(row % D);
  const float* xr = x + row * (long long)S;
  float acc = __ldg(bias + d);
  for (int k = 0; k < W; ++k) {
    const int ts = t - (W - 1) + k;
    if (ts >= 0) acc = fmaf(__ldg(xr + ts), __ldg(w + (long long)d * W + k), acc);
  }
  out[i] = SILU ? silu_f(acc) : acc;
}

// ---------------------------------------------------------------------------
// BSD (channel-last), fp32 or bf16, D % 4 == 0. One thread = 4 channels.
// ---------------------------------------------------------------------------
template <typename T>
struct Vec4;
template <>
struct Vec4<__nv_bfloat16> {
  uint2 raw;
  __device__ __forceinline__ void load(const __nv_bfloat16* p) { raw = __ldg(reinterpret_cast<const uint2*>(p)); }
  __device__ __forceinline__ void to_float(float* f) const {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
    float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  }
  __device__ __forceinline__ static void store(__nv_bfloat16* p, const float* f) {
    uint2 r;
    r.x = pack_bf16x2(f[0], f[1]);
    r.y = pack_bf16x2(f[2], f[3]);
    *reinterpret_cast<uint2*>(p) = r;
  }
  __device__ __forceinline__ void raw_from_smem(const uint8_t* p) { raw = *reinterpret_cast<const uint2*>(p); }
  __device__ __forceinline__ static void store_smem(uint8_t* p, const float* f) {
    store(reinterpret_cast<__nv_bfloat16*>(p), f);
  }
};
template <>
struct Vec4<float> {
  float4 a;
  __device__ __forceinline__ void load(const float* p) { a = ldg4(p); }
  __device__ __forceinline__ void to_float(float* f) const { f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; }
  __device__ __forceinline__ static void store(float* p, const float* f) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  }
  __device__ __forceinline__ void raw_from_smem(const uint8_t* p) { a = *reinterpret_cast<const float4*>(p); }
  __device__ __forceinline__ static void store_smem(uint8_t* p, const float* f) {
    store(reinterpret_cast<float*>(p), f);
  }
};

constexpr int kBsdThreads = 128;
constexpr int kBsdCh = 4;       // channels per thread
constexpr int kBsdTile = 8;     // rows per pipelined tile
constexpr int kBsdStrip = 256;  // time steps per thread strip

// One pipelined tile: rows t_first .. t_first+tt-1 from registers `rows`.
// GL = lanes per L2-norm group (G / 4), 0 = no norm.
template <typename T, int W, bool SILU, int GL>
__device__ __forceinline__ void bsd_tile(Vec4<T>* rows, float (*hist)[kBsdCh], const float (*wr)[W],
                                         const float* bsv, T* ob, int t_first, int S, int D, bool active, int tt) {
#pragma unroll
  for (int i = 0; i < kBsdTile; ++i) {
    if (i >= tt) break;
    const int t = t_first + i;
    float cur[kBsdCh];
    rows[i].to_float(cur);
    float o[kBsdCh];
#pragma unroll
    for (int j = 0; j < kBsdCh; ++j) {
      float acc = bsv[j];
#pragma unroll
      for (int k = 0; k < W - 1; ++k) acc = fmaf(hist[k][j], wr[j][k], acc);
      acc = fmaf(cur[j], wr[j][W - 1], acc);
      o[j] = SILU ? silu_f(acc) : acc;
    }
#pragma unroll
    for (int k = 0; k + 1 < W - 1; ++k)
#pragma unroll
      for (int j = 0; j < kBsdCh; ++j) hist[k][j] = hist[k + 1][j];
    if (W > 1) {
#pragma unroll
      for (int j = 0; j < kBsdCh; ++j) hist[W > 1 ? W - 2 : 0][j] = cur[j];
    }
    if (GL > 0) {
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < kBsdCh; ++j) ss = fmaf(o[j], o[j], ss);
#pragma unroll
      for (int m = 1; m < GL; m <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
      const float r = rsqrtf(ss + 1e-6f);
#pragma unroll
      for (int j = 0; j < kBsdCh; ++j) o[j] *= r;
    }
    if (t < S && active) Vec4<T>::store(ob + (long long)t * D, o);
  }
}

template <typename T>
__device__ __forceinline__ void bsd_load_tile(Vec4<T>* rows, const T* xb, int t_first, int S, int D, bool active) {
#pragma unroll
  for (int i = 0; i < kBsdTile; ++i) {
    const int t = t_first + i;
    if (t < S && active) rows[i].load(xb + (long long)t * D);
  }
}

// A thread owns 4 channels over a 256-step time strip: tile i+1's rows are
// loaded while tile i is computed and stored, and the W-1 previous rows are
// carried in registers (only the strip start re-reads a halo).
template <typename T, int W, bool SILU, int GL>
__global__ void __launch_bounds__(kBsdThreads, 4) conv_bsd(const T* __restrict__ x, const float* __restrict__ w,
                                                           const float* __restrict__ bias, T* __restrict__ out,
                                                           int S, int D) {
  const int c0 = (blockIdx.x * kBsdThreads + threadIdx.x) * kBsdCh;
  const bool active = c0 < D;
  const int cc = active ? c0 : 0;  // keep addresses valid for inactive lanes
  const int t_begin = blockIdx.y * kBsdStrip;
  const int t_end = min(S, t_begin + kBsdStrip);
  const long long bbase = (long long)blockIdx.z * S * D;
  const T* xb = x + bbase + cc;
  T* ob = out + bbase + cc;

  float wr[kBsdCh][W];
  float bsv[kBsdCh];
#pragma unroll
  for (int j = 0; j < kBsdCh; ++j) {
    bsv[j] = __ldg(bias + cc + j);
#pragma unroll
    for (int k = 0; k < W; ++k) wr[j][k] = __ldg(w + (long long)(cc + j) * W + k);
  }
  float hist[W > 1 ? W - 1 : 1][kBsdCh];
#pragma unroll
  for (int k = 0; k < W - 1; ++k) {
    const int ts = t_begin - (W - 1) + k;
    if (ts >= 0 && active) {
      Vec4<T> v;
      v.load(xb + (long long)ts * D);
      v.to_float(hist[k]);
    } else {
#pragma unroll
      for (int j = 0; j < kBsdCh; ++j) hist[k][j] = 0.f;
    }
  }

  Vec4<T> ra[kBsdTile], rb[kBsdTile];
  bsd_load_tile<T>(ra, xb, t_begin, S, D, active);
#pragma unroll 1
  for (int t = t_begin; t < t_end; t += 2 * kBsdTile) {
    if (t + kBsdTile < t_end) bsd_load_tile<T>(rb, xb, t + kBsdTile, S, D, active);
    bsd_tile<T, W, SILU, GL>(ra, hist, wr, bsv, ob, t, S, D, active, min(kBsdTile, t_end - t));
    if (t + kBsdTile < t_end) {
      if (t + 2 * kBsdTile < t_end) bsd_load_tile<T>(ra, xb, t + 2 * kBsdTile, S, D, active);
      bsd_tile<T, W, SILU, GL>(rb, hist, wr, bsv, ob, t + kBsdTile, S, D, active,
                               min(kBsdTile, t_end - t - kBsdTile));
    }
  }
}

// Runtime-W channel-last fallback (W not in {2,3,4}): one thread = 4 channels x 1 step.
template <typename T, bool SILU, int GL>
__global__ void __launch_bounds__(kBsdThreads) conv_bsd_generic(const T* __restrict__ x,
                                                                const float* __restrict__ w,
                                                                const float* __restrict__ bias,
                                                                T* __restrict__ out, int S, int D, int W) {
  const int c0 = (blockIdx.x * kBsdThreads + threadIdx.x) * kBsdCh;
  const bool active = c0 < D;
  const int cc = active ? c0 : 0;
  const int t = blockIdx.y;
  const long long bbase = (long long)blockIdx.z * S * D;
  float o[kBsdCh];
#pragma unroll
  for (int j = 0; j < kBsdCh; ++j) o[j] = __ldg(bias + cc + j);
  for (int k = 0; k < W; ++k) {
    const int ts = t - (W - 1) + k;
    if (ts < 0 || !active) continue;
    Vec4<T> v;
    v.load(x + bbase + (long long)ts * D + cc);
    float f[kBsdCh];
    v.to_float(f);
#pragma unroll
    for (int j = 0; j < kBsdCh; ++j) o[j] = fmaf(f[j], __ldg(w + (long long)(cc + j) * W + k), o[j]);
  }
#pragma unroll
  for (int j = 0; j < kBsdCh; ++j) o[j] = SILU ? silu_f(o[j]) : o[j];
  if (GL > 0) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kBsdCh; ++j) ss = fmaf(o[j], o[j], ss);
#pragma unroll
    for (int m = 1; m < GL; m <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
    const float r = rsqrtf(ss + 1e-6f);
#pragma unroll
    for (int j = 0; j < kBsdCh; ++j) o[j] *= r;
  }
  if (active) Vec4<T>::store(out + bbase + (long long)t * D + cc, o);
}

// ---------------------------------------------------------------------------
// BSD through TMA tiles (D * sizeof(T) % 16 == 0, W <= 8): one CTA = 256
// channels x a strip of STRIP steps (256, or 512 for large grids: see
// long_strips), tiles of 32 rows. Each tile and its W-1 halo
// rows arrive by TMA from a per-batch 3-D map [B][S][D] (rows before t = 0 are
// the map's zero fill), 3-stage ring; the output tile is staged in smem and
// written by TMA store. 256 threads: thread = 4 channels x 8 rows; a warp
// covers 128 consecutive channels of one row group, so a per-head L2 norm of
// up to 128 channels is a warp shuffle reduction.
// ---------------------------------------------------------------------------
namespace tma {
constexpr int kThreads = 256;
constexpr int kCh = 256;     // channels per CTA
constexpr int kRows = 32;    // output rows per tile
constexpr int kStrip = 256;  // rows per CTA (kLongStrip for large grids)
constexpr int kLongStrip = 512;
constexpr int kStages = 2;

template <typename T, int W>
struct Layout {
  static constexpr int ES = sizeof(T);
  static constexpr int IN_ROWS = kRows + W - 1;
  static constexpr int IN_BYTES = IN_ROWS * kCh * ES;
  static constexpr int IN_STRIDE = (IN_BYTES + 1023) / 1024 * 1024;
  static constexpr int OUT_BYTES = kRows * kCh * ES;
  static constexpr int OFF_OUT = kStages * IN_STRIDE;
  static constexpr int OFF_BAR = OFF_OUT + 2 * OUT_BYTES;
  static constexpr int SMEM = OFF_BAR + 64 + 1024;
};

// Strip length for a launch. Each CTA pays a fixed start (barriers, weights,
// the first TMA round trip), so longer strips stream more bytes per start; but a
// grid of few waves (3 CTAs per SM) loses more to its last, partly filled wave
// than it saves. Measured at T = 8192, D = 2048, bf16 (µs for one conv):
// B = 16: 191.7 with 256-row strips, 185.6 with 512, 187.6 with 1024;
// B = 8: 100.7 / 98.8 / 111.2; B = 4: 54.4 / 59.9 / 60.2; B = 2: 33.6 / 33.6 / 42.0.
// So 512 rows where that grid still fills at least two waves, else 256.
inline bool long_strips(int B, int D, int S) {
  const long long ctas = (long long)((D + kCh - 1) / kCh) * B * ((S + kLongStrip - 1) / kLongStrip);
  return ctas >= 2LL * 3 * sm_count();
}

// One row of the thread's 4 channels: shared memory <-> fp32 registers.
template <typename T>
__device__ __forceinline__ void load_row(const uint8_t* p, float* f) {
  if constexpr (sizeof(T) == 2) {
    const uint2 r = *reinterpret_cast<const uint2*>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.x));
    const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.y));
    f[0] = a.x; f[1] = a.y; f[2] = c.x; f[3] = c.y;
  } else {
    const float4 a = *reinterpret_cast<const float4*>(p);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  }
}

template <typename T>
__device__ __forceinline__ void store_row(uint8_t* p, const float* f) {
  if constexpr (sizeof(T) == 2) {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]));
  } else {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  }
}

// silu for bf16 outputs: x sigmoid(x) = h + h tanh(h), h = x/2, with the
// hardware tanh approximation (relative error ~2^-11, below bf16's 2^-9
// output rounding). fp32 outputs keep silu_f.
__device__ __forceinline__ float silu_tanh(float x) {
  const float h = 0.5f * x;
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(h));
  return fmaf(h, t, h);
}

// One CTA's strip of one sequence b (the body of both kernels below).
template <typename T, int W, bool SILU, int GL, int STRIP>
__device__ __forceinline__ void bsd_tma_strip(const CUtensorMap* tm_x, const CUtensorMap* tm_o,
                                              const float* __restrict__ w, const float* __restrict__ bias, int S,
                                              int D, int b) {
  using Ly = Layout<T, W>;
  constexpr int C = 4;                           // channels per thread
  constexpr int NCG = kCh / C;                   // channel groups across the 256 channels
  constexpr int RPT = kRows / (kThreads / NCG);  // rows per thread per tile (8)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + Ly::OFF_BAR);
  const int tid = threadIdx.x;
  const int cg = tid % NCG, rq = tid / NCG;  // channel group, row band
  const int c0 = blockIdx.x * kCh;
  const int t_begin = blockIdx.y * STRIP;
  const int ntiles = min(STRIP, S - t_begin + kRows - 1) / kRows;
  const int cc = min(c0 + C * cg, D - C);  // clamp: channels past D are computed but not stored

  float wr[C][W], bs[C];
#pragma unroll
  for (int j = 0; j < C; ++j) {
    bs[j] = __ldg(bias + cc + j);
#pragma unroll
    for (int k = 0; k < W; ++k) wr[j][k] = __ldg(w + (long long)(cc + j) * W + k);
  }
  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) mbar_init(&full[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int i) {
    const int st = i % kStages;
    mbar_arrive_expect_tx(&full[st], Ly::IN_ROWS * kCh * Ly::ES);
    tma_load_3d(sm + st * Ly::IN_STRIDE, tm_x, &full[st], c0, t_begin + i * kRows - (W - 1), b);
  };
  if (tid == 0)
    for (int i = 0; i < kStages && i < ntiles; ++i) issue(i);

  bool ok = true;
  for (int i = 0; i < ntiles; ++i) {
    const int st = i % kStages, ob = i & 1;
    // the store that last used this output buffer (tile i-2) has read it
    if (tid == 0 && i >= 2) bulk_wait_group_read1();
    ok = mbar_wait(&full[st], (i / kStages) & 1, &g_status_conv);
    ok = __syncthreads_and(ok);
    if (!ok) break;
    const uint8_t* in = sm + st * Ly::IN_STRIDE;
    uint8_t* out = sm + Ly::OFF_OUT + ob * Ly::OUT_BYTES;
    // rows r0-W+1 .. r0+RPT-1 of this band (smem row = tile row + W - 1)
    float xr[RPT + W - 1][C];
#pragma unroll
    for (int j = 0; j < RPT + W - 1; ++j) load_row<T>(in + ((RPT * rq + j) * kCh + C * cg) * Ly::ES, xr[j]);
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
      // channel pairs as packed fp32x2 (each lane an fmaf / fmul of the same
      // operands as the scalar form, so the results are unchanged)
      float o[C];
#pragma unroll
      for (int j = 0; j < C; j += 2) {
        float2 acc = make_float2(bs[j], bs[j + 1]);
#pragma unroll
        for (int k = 0; k < W; ++k)
          acc = __ffma2_rn(make_float2(xr[r + k][j], xr[r + k][j + 1]), make_float2(wr[j][k], wr[j + 1][k]), acc);
        if (SILU && sizeof(T) == 2) {
          // silu_tanh on the pair: h + h tanh(h), h = x / 2
          const float2 h = __fmul2_rn(make_float2(0.5f, 0.5f), acc);
          float t0, t1;
          asm("tanh.approx.f32 %0, %1;" : "=f"(t0) : "f"(h.x));
          asm("tanh.approx.f32 %0, %1;" : "=f"(t1) : "f"(h.y));
          const float2 sv = __ffma2_rn(h, make_float2(t0, t1), h);
          o[j] = sv.x;
          o[j + 1] = sv.y;
        } else {
          o[j] = SILU ? silu_f(acc.x) : acc.x;
          o[j + 1] = SILU ? silu_f(acc.y) : acc.y;
        }
      }
      if (GL > 0) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < C; ++j) ss = fmaf(o[j], o[j], ss);
#pragma unroll
        for (int m = 1; m < GL; m <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
        const float rn = rsqrtf(ss + 1e-6f);
#pragma unroll
        for (int j = 0; j < C; j += 2) {
          const float2 sc2 = __fmul2_rn(make_float2(o[j], o[j + 1]), make_float2(rn, rn));
          o[j] = sc2.x;
          o[j + 1] = sc2.y;
        }
      }
      store_row<T>(out + ((RPT * rq + r) * kCh + C * cg) * Ly::ES, o);
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      tma_store_3d(tm_o, out, c0, t_begin + i * kRows, b);
      bulk_commit_group();
      if (i + kStages < ntiles) issue(i + kStages);
    }
  }
  if (tid == 0) bulk_wait_group0();
}

template <typename T, int W, bool SILU, int GL, int STRIP>
__global__ void __launch_bounds__(kThreads, 3)
    conv_bsd_tma(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_o,
                 const float* __restrict__ w, const float* __restrict__ bias, int S, int D) {
  bsd_tma_strip<T, W, SILU, GL, STRIP>(&tm_x, &tm_o, w, bias, S, D, blockIdx.z);
}

// Two convs of the same shape in one grid (the layer's q and k projections):
// blockIdx.z < B is sequence z of the first, else sequence z - B of the second.
// One grid of 2B sequences has half as many partly filled last waves as two
// launches of B, which matters when B is small.
template <typename T, int W, bool SILU, int GL, int STRIP>
__global__ void __launch_bounds__(kThreads, 3)
    conv_bsd_tma_pair(const __grid_constant__ CUtensorMap tm_x0, const __grid_constant__ CUtensorMap tm_o0,
                      const float* __restrict__ w0, const float* __restrict__ bias0,
                      const __grid_constant__ CUtensorMap tm_x1, const __grid_constant__ CUtensorMap tm_o1,
                      const float* __restrict__ w1, const float* __restrict__ bias1, int S, int D, int B) {
  const bool second = (int)blockIdx.z >= B;
  bsd_tma_strip<T, W, SILU, GL, STRIP>(second ? &tm_x1 : &tm_x0, second ? &tm_o1 : &tm_o0, second ? w1 : w0,
                                       second ? bias1 : bias0, S, D, (int)blockIdx.z - (second ? B : 0));
}
}  // namespace tma

// ---------------------------------------------------------------------------
// dispatch
// ---------------------------------------------------------------------------
template <int W, bool SILU>
void launch_bds_vec(const float* x, const float* w, const float* b, float* o, int B, int D, int S,
                    cudaStream_t st) {
  if constexpr (W <= 5) {
    const dim3 grid((unsigned)(B * D), (unsigned)((S / 4 + kBdsQ - 1) / kBdsQ));
    conv_bds_f4<W, SILU><<<grid, kBdsThreads, 0, st>>>(x, w, b, o, D, S);
  } else {
    const int nseg_row = (S + 7) / 8;
    const long long total = (long long)B * D * nseg_row;
    conv_bds_vec8<W, SILU><<<(unsigned)((total + 255) / 256), 256, 0, st>>>(x, w, b, o, D, S, total, nseg_row);
  }
}

template <bool SILU>
int dispatch_bds(const float* x, const float* w, const float* b, float* o, int B, int D, int S, int W,
                 cudaStream_t st) {
  const bool grid_ok = W > 5 || ((long long)B * D <= 0x7fffffffLL && (S / 4 + kBdsQ - 1) / kBdsQ <= 65535);
  const bool vec = (S % 4 == 0) && W <= 8 && aligned16(x) && aligned16(o) && grid_ok;
  if (!vec) {
    const long long total = (long long)B * D * S;
    conv_bds_scalar<SILU><<<(unsigned)((total + 255) / 256), 256, 0, st>>>(x, w, b, o, D, S, W, total);
    return check_launch();
  }
  switch (W) {
    case 1: launch_bds_vec<1, SILU>(x, w, b, o, B, D, S, st); break;
    case 2: launch_bds_vec<2, SILU>(x, w, b, o, B, D, S, st); break;
    case 3: launch_bds_vec<3, SILU>(x, w, b, o, B, D, S, st); break;
    case 4: launch_bds_vec<4, SILU>(x, w, b, o, B, D, S, st); break;
    case 5: launch_bds_vec<5, SILU>(x, w, b, o, B, D, S, st); break;
    case 6: launch_bds_vec<6, SILU>(x, w, b, o, B, D, S, st); break;
    case 7: launch_bds_vec<7, SILU>(x, w, b, o, B, D, S, st); break;
    default: launch_bds_vec<8, SILU>(x, w, b, o, B, D, S, st); break;
  }
  return check_launch();
}

template <typename T, int W, bool SILU, int GL>
void launch_bsd(const T* x, const float* w, const float* b, T* o, int B, int D, int S, cudaStream_t st) {
  dim3 grid((D / kBsdCh + kBsdThreads - 1) / kBsdThreads, (S + kBsdStrip - 1) / kBsdStrip, B);
  conv_bsd<T, W, SILU, GL><<<grid, kBsdThreads, 0, st>>>(x, w, b, o, S, D);
}

template <typename T, int W, bool SILU, int GL>
int launch_bsd_tma(const T* x, const float* w, const float* b, T* o, int B, int D, int S, cudaStream_t st) {
  using Ly = tma::Layout<T, W>;
  const CUtensorMapDataType dt = sizeof(T) == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUtensorMap tx, to;
  uint64_t dims[3] = {(uint64_t)D, (uint64_t)S, (uint64_t)B};
  uint64_t str[2] = {(uint64_t)D * sizeof(T), (uint64_t)S * D * sizeof(T)};
  uint32_t ibox[3] = {(uint32_t)tma::kCh, (uint32_t)Ly::IN_ROWS, 1u};
  uint32_t obox[3] = {(uint32_t)tma::kCh, (uint32_t)tma::kRows, 1u};
  int r = encode_tiled(&tx, dt, 3, x, dims, str, ibox, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (r == THM_OK) r = encode_tiled(&to, dt, 3, o, dims, str, obox, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (r != THM_OK) return r;
  const bool lng = tma::long_strips(B, D, S);
  auto kern = lng ? tma::conv_bsd_tma<T, W, SILU, GL, tma::kLongStrip> : tma::conv_bsd_tma<T, W, SILU, GL, tma::kStrip>;
  const int strip = lng ? tma::kLongStrip : tma::kStrip;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Ly::SMEM) != cudaSuccess)
    return THM_ERR_CUDA;
  dim3 grid((D + tma::kCh - 1) / tma::kCh, (S + strip - 1) / strip, B);
  kern<<<grid, tma::kThreads, Ly::SMEM, st>>>(tx, to, w, b, S, D);
  return check_launch();
}

template <typename T, int W, bool SILU, int GL>
int launch_bsd_tma_pair(const T* x0, const float* w0, const float* b0, T* o0, const T* x1, const float* w1,
                        const float* b1, T* o1, int B, int D, int S, cudaStream_t st) {
  using Ly = tma::Layout<T, W>;
  const CUtensorMapDataType dt = sizeof(T) == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUtensorMap tx0, to0, tx1, to1;
  uint64_t dims[3] = {(uint64_t)D, (uint64_t)S, (uint64_t)B};
  uint64_t str[2] = {(uint64_t)D * sizeof(T), (uint64_t)S * D * sizeof(T)};
  uint32_t ibox[3] = {(uint32_t)tma::kCh, (uint32_t)Ly::IN_ROWS, 1u};
  uint32_t obox[3] = {(uint32_t)tma::kCh, (uint32_t)tma::kRows, 1u};
  int r = encode_tiled(&tx0, dt, 3, x0, dims, str, ibox, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (r == THM_OK) r = encode_tiled(&to0, dt, 3, o0, dims, str, obox, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (r == THM_OK) r = encode_tiled(&tx1, dt, 3, x1, dims, str, ibox, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (r == THM_OK) r = encode_tiled(&to1, dt, 3, o1, dims, str, obox, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (r != THM_OK) return r;
  const bool lng = tma::long_strips(2 * B, D, S);
  auto kern = lng ? tma::conv_bsd_tma_pair<T, W, SILU, GL, tma::kLongStrip>
                  : tma::conv_bsd_tma_pair<T, W, SILU, GL, tma::kStrip>;
  const int strip = lng ? tma::kLongStrip : tma::kStrip;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Ly::SMEM) != cudaSuccess)
    return THM_ERR_CUDA;
  dim3 grid((D + tma::kCh - 1) / tma::kCh, (S + strip - 1) / strip, 2 * B);
  kern<<<grid, tma::kThreads, Ly::SMEM, st>>>(tx0, to0, w0, b0, tx1, to1, w1, b1, S, D, B);
  return check_launch();
}

template <typename T, bool SILU, int GL>
int dispatch_bsd_w(const T* x, const float* w, const float* b, T* o, int B, int D, int S, int W,
                   cudaStream_t st) {
  if ((D * (int)sizeof(T)) % 16 == 0 && D >= 4 && (W == 2 || W == 3 || W == 4)) {
    switch (W) {
      case 2: return launch_bsd_tma<T, 2, SILU, GL>(x, w, b, o, B, D, S, st);
      case 3: return launch_bsd_tma<T, 3, SILU, GL>(x, w, b, o, B, D, S, st);
      default: return launch_bsd_tma<T, 4, SILU, GL>(x, w, b, o, B, D, S, st);
    }
  }
  switch (W) {
    case 2: launch_bsd<T, 2, SILU, GL>(x, w, b, o, B, D, S, st); break;
    case 3: launch_bsd<T, 3, SILU, GL>(x, w, b, o, B, D, S, st); break;
    case 4: launch_bsd<T, 4, SILU, GL>(x, w, b, o, B, D, S, st); break;
    default: {
      dim3 grid((D / kBsdCh + kBsdThreads - 1) / kBsdThreads, S, B);
      conv_bsd_generic<T, SILU, GL><<<grid, kBsdThreads, 0, st>>>(x, w, b, o, S, D, W);
    }
  }
  return check_launch();
}

template <typename T, bool SILU>
int dispatch_bsd(const T* x, const float* w, const float* b, T* o, int B, int D, int S, int W, int G,
                 cudaStream_t st) {
  switch (G) {
    case 0: return dispatch_bsd_w<T, SILU, 0>(x, w, b, o, B, D, S, W, st);
    case 16: return dispatch_bsd_w<T, SILU, 4>(x, w, b, o, B, D, S, W, st);
    case 32: return dispatch_bsd_w<T, SILU, 8>(x, w, b, o, B, D, S, W, st);
    case 64: return dispatch_bsd_w<T, SILU, 16>(x, w, b, o, B, D, S, W, st);
    case 128: return dispatch_bsd_w<T, SILU, 32>(x, w, b, o, B, D, S, W, st);
    default: return THM_ERR_UNSUPPORTED;
  }
}

// Both convs in one launch where the TMA path applies (one grid of 2B sequences),
// else as two launches of the single-conv path.
template <typename T, bool SILU, int GL>
int dispatch_bsd_pair_w(const T* x0, const float* w0, const float* b0, T* o0, const T* x1, const float* w1,
                        const float* b1, T* o1, int B, int D, int S, int W, cudaStream_t st) {
  if ((D * (int)sizeof(T)) % 16 == 0 && D >= 4 && (W == 2 || W == 3 || W == 4) && 2LL * B <= 65535) {
    switch (W) {
      case 2: return launch_bsd_tma_pair<T, 2, SILU, GL>(x0, w0, b0, o0, x1, w1, b1, o1, B, D, S, st);
      case 3: return launch_bsd_tma_pair<T, 3, SILU, GL>(x0, w0, b0, o0, x1, w1, b1, o1, B, D, S, st);
      default: return launch_bsd_tma_pair<T, 4, SILU, GL>(x0, w0, b0, o0, x1, w1, b1, o1, B, D, S, st);
    }
  }
  const int r = dispatch_bsd_w<T, SILU, GL>(x0, w0, b0, o0, B, D, S, W, st);
  return r != THM_OK ? r : dispatch_bsd_w<T, SILU, GL>(x1, w1, b1, o1, B, D, S, W, st);
}

template <typename T, bool SILU>
int dispatch_bsd_pair(const T* x0, const float* w0, const float* b0, T* o0, const T* x1, const float* w1,
                      const float* b1, T* o1, int B, int D, int S, int W, int G, cudaStream_t st) {
  switch (G) {
    case 0: return dispatch_bsd_pair_w<T, SILU, 0>(x0, w0, b0, o0, x1, w1, b1, o1, B, D, S, W, st);
    case 16: return dispatch_bsd_pair_w<T, SILU, 4>(x0, w0, b0, o0, x1, w1, b1, o1, B, D, S, W, st);
    case 32: return dispatch_bsd_pair_w<T, SILU, 8>(x0, w0, b0, o0, x1, w1, b1, o1, B, D, S, W, st);
    case 64: return dispatch_bsd_pair_w<T, SILU, 16>(x0, w0, b0, o0, x1, w1, b1, o1, B, D, S, W, st);
    case 128: return dispatch_bsd_pair_w<T, SILU, 32>(x0, w0, b0, o0, x1, w1, b1, o1, B, D, S, W, st);
    default: return THM_ERR_UNSUPPORTED;
  }
}

}  // namespace conv
}  // namespace thm

THM_STATUS_READER(thm_internal_status_conv, g_status_conv)

extern "C" int thm_causal_conv1d_fwd(const void* x, const float* weight, const float* bias, void* out, int B,
                                     int D, int S, int W, int layout, int dtype, int activation,
                                     int l2norm_group, thm_stream_t stream) {
  using namespace thm;
  using namespace thm::conv;
  if (B < 0 || D < 0 || S < 0 || W < 1) return THM_ERR_INVALID;
  if (activation != THM_ACT_NONE && activation != THM_ACT_SILU) return THM_ERR_INVALID;
  if (layout != THM_LAYOUT_BDS && layout != THM_LAYOUT_BSD) return THM_ERR_INVALID;
  if (dtype != THM_F32 && dtype != THM_BF16) return THM_ERR_INVALID;
  if ((long long)B * D * S == 0) return THM_OK;  // empty tensor: nothing to do
  if (!x || !weight || !bias || !out) return THM_ERR_INVALID;
  if (W > 64) return THM_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool silu = activation == THM_ACT_SILU;
  if (layout == THM_LAYOUT_BDS) {
    if (dtype != THM_F32 || l2norm_group != 0) return THM_ERR_UNSUPPORTED;
    const float* xf = static_cast<const float*>(x);
    float* of = static_cast<float*>(out);
    return silu ? dispatch_bds<true>(xf, weight, bias, of, B, D, S, W, st)
                : dispatch_bds<false>(xf, weight, bias, of, B, D, S, W, st);
  }
  if (D % 4 != 0) return THM_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(out)) return THM_ERR_ALIGNMENT;
  if (l2norm_group != 0 && D % l2norm_group != 0) return THM_ERR_INVALID;
  if (dtype == THM_BF16) {
    auto xb = static_cast<const __nv_bfloat16*>(x);
    auto ob = static_cast<__nv_bfloat16*>(out);
    return silu ? dispatch_bsd<__nv_bfloat16, true>(xb, weight, bias, ob, B, D, S, W, l2norm_group, st)
                : dispatch_bsd<__nv_bfloat16, false>(xb, weight, bias, ob, B, D, S, W, l2norm_group, st);
  }
  auto xf = static_cast<const float*>(x);
  auto of = static_cast<float*>(out);
  return silu ? dispatch_bsd<float, true>(xf, weight, bias, of, B, D, S, W, l2norm_group, st)
              : dispatch_bsd<float, false>(xf, weight, bias, of, B, D, S, W, l2norm_group, st);
}

extern "C" int thm_causal_conv1d_pair_fwd(const void* x0, const float* weight0, const float* bias0, void* out0,
                                          const void* x1, const float* weight1, const float* bias1, void* out1,
                                          int B, int D, int S, int W, int dtype, int activation, int l2norm_group,
                                          thm_stream_t stream) {
  using namespace thm;
  using namespace thm::conv;
  if (B < 0 || D < 0 || S < 0 || W < 1) return THM_ERR_INVALID;
  if (activation != THM_ACT_NONE && activation != THM_ACT_SILU) return THM_ERR_INVALID;
  if (dtype != THM_F32 && dtype != THM_BF16) return THM_ERR_INVALID;
  if ((long long)B * D * S == 0) return THM_OK;  // empty tensors: nothing to do
  if (!x0 || !weight0 || !bias0 || !out0 || !x1 || !weight1 || !bias1 || !out1) return THM_ERR_INVALID;
  if (W > 64) return THM_ERR_UNSUPPORTED;
  if (D % 4 != 0) return THM_ERR_UNSUPPORTED;
  if (!aligned16(x0) || !aligned16(out0) || !aligned16(x1) || !aligned16(out1)) return THM_ERR_ALIGNMENT;
  if (l2norm_group != 0 && D % l2norm_group != 0) return THM_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool silu = activation == THM_ACT_SILU;
  if (dtype == THM_BF16) {
    using bf = __nv_bfloat16;
    auto a0 = static_cast<const bf*>(x0);
    auto a1 = static_cast<const bf*>(x1);
    auto p0 = static_cast<bf*>(out0);
    auto p1 = static_cast<bf*>(out1);
    return silu ? dispatch_bsd_pair<bf, true>(a0, weight0, bias0, p0, a1, weight1, bias1, p1, B, D, S, W, l2norm_group, st)
                : dispatch_bsd_pair<bf, false>(a0, weight0, bias0, p0, a1, weight1, bias1, p1, B, D, S, W, l2norm_group, st);
  }
  auto a0 = static_cast<const float*>(x0);
  auto a1 = static_cast<const float*>(x1);
  auto p0 = static_cast<float*>(out0);
  auto p1 = static_cast<float*>(out1);
  return silu ? dispatch_bsd_pair<float, true>(a0, weight0, bias0, p0, a1, weight1, bias1, p1, B, D, S, W, l2norm_group, st)
              : dispatch_bsd_pair<float, false>(a0, weight0, bias0, p0, a1, weight1, bias1, p1, B, D, S, W, l2norm_group, st);
}
