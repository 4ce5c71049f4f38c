// recompute_w_u.cu -- gated-DeltaNet WY recompute of (w, u) on tcgen05.
//
// Replaces kernels/recompute_w_u/kernel.py:73-186 (recompute_w_u_kernel) and
// its launcher :192-248. One CTA per (b, h, 64-token chunk), 128 threads:
//
//   k, v tiles ------------------------------------------- TMA (swizzled)
//   [a_mode != 0]  KK^T (M=64, N=64, K=K) on the tensor core -> TMEM
//                  M_ij = beta_i k_i.k_j exp(g_i - g_j), j < i     registers
//                  A = (I + sign*M)^-1 by column-parallel forward substitution
//                  in shared memory (thread j owns column j)
//   [a_mode == 0]  A by TMA (fp32, K-major)
//   k <- k * beta * exp(g), v <- v * beta   row scaling in shared memory
//   W = A k   (M=64, N=K, K=64),  U = A v   (M=64, N=V, K=64)  tensor core
//   TMEM -> registers -> w, u in HBM
//
// sign = -1 is the reference's upstream producer (I - M)^-1
// (kernels/recompute_w_u/reference.py:48-91); sign = +1 the gated-DeltaNet
// (I + M)^-1. bf16 operands use kind::f16, fp32 operands kind::tf32 (KK^T in
// 3xTF32, so the fp32 A matches an fp32 solve); all accumulation is fp32 in
// TMEM.
#include <cuda_bf16.h>

#include "host_util.h"
#include "sm100.cuh"

THM_DEFINE_STATUS(g_status_wu)

namespace thm {
namespace wu {

constexpr int kThreads = 128;
constexpr int kBT = 64;

template <typename T, int K, int V>
struct Layout {
  static constexpr int ES = sizeof(T);
  static constexpr bool BF16 = ES == 2;
  static constexpr int K_BYTES = kBT * K * ES;    // k tile, MN-major B operand of W
  static constexpr int KK_BYTES = BF16 ? 0 : kBT * K * ES;  // fp32: K-major copy for KK^T (hi)
  static constexpr int KKLO_BYTES = KK_BYTES;               // fp32: its lo part (3xTF32)
  static constexpr int V_BYTES = kBT * V * ES;
  static constexpr int AF_BYTES = kBT * kBT * 4;  // A fp32 (TMA target; fp32 path's MMA operand)
  static constexpr int A16_BYTES = BF16 ? kBT * kBT * 2 : 0;  // A bf16 (MMA operand, bf16 path)
  static constexpr int M_BYTES = kBT * kBT * 4;   // strictly lower M, fp32 (fused solve)
  static constexpr int OFF_K = 0;
  static constexpr int OFF_KK = OFF_K + K_BYTES;
  static constexpr int OFF_KKLO = OFF_KK + KK_BYTES;
  static constexpr int OFF_V = OFF_KKLO + KKLO_BYTES;
  static constexpr int OFF_AF = OFF_V + V_BYTES;
  static constexpr int OFF_A16 = OFF_AF + AF_BYTES;
  static constexpr int OFF_M = OFF_A16 + A16_BYTES;
  static constexpr int OFF_MISC = OFF_M + M_BYTES;
  static constexpr int SMEM = OFF_MISC + 2048 + 1024;
  static constexpr uint32_t TMEM_COLS = (K + V) <= 128 ? 128 : 256;  // W [0,K) | U [K,K+V)
};

template <typename T, int K, int V>
__global__ void __launch_bounds__(kThreads, 1)
    recompute_w_u_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_kk,
                         const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_a,
                         const float* __restrict__ beta, const float* __restrict__ g, T* __restrict__ w,
                         T* __restrict__ u, float* __restrict__ a_out, int T_len, int H, int a_mode) {
  using Ly = Layout<T, K, V>;
  constexpr bool kBf16 = Ly::BF16;
  constexpr uint32_t kFmt = kBf16 ? 1u : 2u;
  constexpr int kStep = kBf16 ? 16 : 8;
  constexpr uint32_t kIdKK = make_idesc(kFmt, 64, 64, 0, 0);
  constexpr uint32_t kIdW = make_idesc(kFmt, 64, K, 0, 1);
  constexpr uint32_t kIdU = make_idesc(kFmt, 64, V, 0, 1);
  // MN-major B operand (k, v): bf16 -> SW128 (8-row atoms); tf32 -> 32-B atoms.
  constexpr uint32_t kBLayout = kBf16 ? kSw128 : kSw128Base32;
  constexpr uint32_t kBSbo = kBf16 ? 1024u : 512u;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(sm);
  float* sBeta = reinterpret_cast<float*>(sm + Ly::OFF_MISC);  // 64
  float* sG = sBeta + 64;                                        // 64
  float* sFk = sG + 64;                                          // beta*exp(g)
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(sm + Ly::OFF_MISC + 1024);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_tma + 2);
  float(*sM)[kBT] = reinterpret_cast<float(*)[kBT]>(sm + Ly::OFF_M);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int row0 = b * T_len + c * kBT;
  const bool fused = a_mode != 0;
  uint32_t mma_phase = 0;
  int pending = -1;  // parity of an MMA commit not yet waited for (cleanup path)

  if (tid == 0) {
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, Ly::TMEM_COLS);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tW = tbase, tU = tbase + K;

  if (tid == 0) {
    constexpr int kBox = 128 / Ly::ES;
    uint32_t bytes = Ly::K_BYTES + Ly::V_BYTES + (fused ? Ly::KK_BYTES : Ly::AF_BYTES);
    mbar_arrive_expect_tx(bar_tma, bytes);
#pragma unroll
    for (int j = 0; j < K / kBox; ++j) {
      tma_load_3d(sm + Ly::OFF_K + j * kBT * 128, &tm_k, bar_tma, j * kBox, h, row0);
      if (!kBf16 && fused) tma_load_3d(sm + Ly::OFF_KK + j * kBT * 128, &tm_kk, bar_tma, j * kBox, h, row0);
    }
#pragma unroll
    for (int j = 0; j < V / kBox; ++j) tma_load_3d(sm + Ly::OFF_V + j * kBT * 128, &tm_v, bar_tma, j * kBox, h, row0);
    if (!fused) {
      tma_load_3d(sm + Ly::OFF_AF, &tm_a, bar_tma, 0, h, row0);
      tma_load_3d(sm + Ly::OFF_AF + kBT * 128, &tm_a, bar_tma, 32, h, row0);
    }
  }
  if (tid < kBT) {
    const long long gi = (long long)(row0 + tid) * H + h;
    const float bv = beta[gi], gv = g[gi];
    sBeta[tid] = bv;
    sG[tid] = gv;
    sFk[tid] = bv * expf(gv);
  }

  bool ok = mbar_wait(bar_tma, 0, &g_status_wu);
  ok = __syncthreads_and(ok);
  if (!ok) goto cleanup;

  if (fused) {
    // KK^T on the tensor core (raw k, K-major view); fp32 operands in 3xTF32.
    if constexpr (!kBf16) {
      split_tf32_tile(sm + Ly::OFF_KK, sm + Ly::OFF_KKLO, Ly::KK_BYTES, tid, kThreads);
      fence_proxy_async_smem();
      __syncthreads();
    }
    if (tid == 0) {
      tc_fence_after();
      constexpr uint32_t kKKOff = kBf16 ? Ly::OFF_K : Ly::OFF_KK;
#pragma unroll
      for (int kk = 0; kk < K / kStep; ++kk) {
        const uint32_t kb = kk * 32;
        const uint32_t off = (kb / 128) * (kBT * 128) + (kb % 128);
        const uint64_t d = make_sdesc(sbase + kKKOff + off, 16, 1024);
        mma_kind<kBf16>(tW, d, d, kIdKK, kk > 0);
        if constexpr (!kBf16) {
          const uint64_t dl = make_sdesc(sbase + Ly::OFF_KKLO + off, 16, 1024);
          mma_tf32_ss(tW, d, dl, kIdKK, 1);
          mma_tf32_ss(tW, dl, d, kIdKK, 1);
        }
      }
      mma_commit(bar_mma);
    }
    pending = (int)mma_phase;
    ok = mbar_wait(bar_mma, mma_phase, &g_status_wu);
    mma_phase ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) goto cleanup;
    pending = -1;
    tc_fence_after();
    {
      // M_ij = beta_i (k_i.k_j) exp(g_i - g_j) for j < i, else 0.
      const int i = warp * 16 + lane;
      const uint32_t la = tW + ((uint32_t)(warp * 32) << 16);
#pragma unroll
      for (int j0 = 0; j0 < kBT; j0 += 32) {
        float s[32];
        tmem_ld32(la + j0, s);
        if (lane < 16) {
          const float bi = sBeta[i], gi = sG[i];
#pragma unroll
          for (int jj = 0; jj < 32; jj += 4) {
            float4 m4;
            float* mv = reinterpret_cast<float*>(&m4);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int j = j0 + jj + q;
              mv[q] = (j < i) ? bi * s[jj + q] * __expf(gi - sG[j]) : 0.0f;
            }
            *reinterpret_cast<float4*>(&sM[i][j0 + jj]) = m4;
          }
        }
      }
    }
    tc_fence_before();
    __syncthreads();
  }

  // Warps 0-1: the triangular solve (fused) or nothing; warps 2-3 scale k, v.
  if (fused && tid < kBT) {
    const int j = tid;
    const float sgn = (a_mode > 0) ? 1.0f : -1.0f;
    float x[kBT];
#pragma unroll
    for (int i = 0; i < kBT; ++i) x[i] = 0.0f;
#pragma unroll
    for (int i = 0; i < kBT; ++i) {
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
      for (int m = 0; m < i; m += 4) {
        const float4 mv = *reinterpret_cast<const float4*>(&sM[i][m]);
        s0 = fmaf(mv.x, x[m], s0);
        s1 = fmaf(mv.y, x[m + 1], s1);
        s2 = fmaf(mv.z, x[m + 2], s2);
        s3 = fmaf(mv.w, x[m + 3], s3);
      }
      x[i] = ((i == j) ? 1.0f : 0.0f) - sgn * ((s0 + s1) + (s2 + s3));
    }
    // x[i] = A[i][j]: write column j of A as the MMA's K-major A operand.
#pragma unroll
    for (int i = 0; i < kBT; ++i) {
      if constexpr (kBf16)
        *reinterpret_cast<__nv_bfloat16*>(sm + Ly::OFF_A16 + sw128_offset(i, j, kBT, 2)) = __float2bfloat16_rn(x[i]);
      else
        *reinterpret_cast<float*>(sm + Ly::OFF_AF + sw128_offset(i, j, kBT, 4)) = x[i];
    }
    if (a_out != nullptr) {
#pragma unroll
      for (int i = 0; i < kBT; ++i) a_out[((long long)(row0 + i) * H + h) * kBT + j] = x[i];
    }
  } else if (!fused || tid >= kBT) {
    const int t0 = fused ? tid - kBT : tid;
    const int nt = fused ? kThreads - kBT : kThreads;
    scale_rows<T>(sm + Ly::OFF_K, K, sFk, t0, nt);
    scale_rows<T>(sm + Ly::OFF_V, V, sBeta, t0, nt);
    if (!fused && kBf16) {
      // A (fp32, TMA) -> bf16 K-major operand.
      for (int i = t0; i < kBT * kBT / 8; i += nt) {
        const int r = i / 8, c0 = (i % 8) * 8;
        float f[8];
#pragma unroll
        for (int q = 0; q < 8; q += 4)
          *reinterpret_cast<float4*>(f + q) =
              *reinterpret_cast<const float4*>(sm + Ly::OFF_AF + sw128_offset(r, c0 + q, kBT, 4));
        uint4 p;
        p.x = pack_bf16x2(f[0], f[1]);
        p.y = pack_bf16x2(f[2], f[3]);
        p.z = pack_bf16x2(f[4], f[5]);
        p.w = pack_bf16x2(f[6], f[7]);
        *reinterpret_cast<uint4*>(sm + Ly::OFF_A16 + sw128_offset(r, c0, kBT, 2)) = p;
      }
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();

  if (tid == 0) {
    tc_fence_after();
    constexpr uint32_t kAOff = kBf16 ? Ly::OFF_A16 : Ly::OFF_AF;
#pragma unroll
    for (int kk = 0; kk < kBT / kStep; ++kk) {
      const uint32_t kb = kk * 32;
      const uint64_t ad = make_sdesc(sbase + kAOff + (kb / 128) * (kBT * 128) + (kb % 128), 16, 1024);
      const uint32_t brow = kk * kStep * 128;
      mma_kind<kBf16>(tW, ad, make_sdesc(sbase + Ly::OFF_K + brow, kBT * 128, kBSbo, kBLayout), kIdW, kk > 0);
      mma_kind<kBf16>(tU, ad, make_sdesc(sbase + Ly::OFF_V + brow, kBT * 128, kBSbo, kBLayout), kIdU, kk > 0);
    }
    mma_commit(bar_mma);
  }
  pending = (int)mma_phase;
  ok = mbar_wait(bar_mma, mma_phase, &g_status_wu);
  mma_phase ^= 1;
  ok = __syncthreads_and(ok);
  if (!ok) goto cleanup;
  pending = -1;
  tc_fence_after();

  {
    const int t = warp * 16 + lane;
    const uint32_t la = (uint32_t)(warp * 32) << 16;
    const long long orow = (long long)(row0 + (lane < 16 ? t : 0)) * H + h;
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      const int n = part == 0 ? K : V;
      const uint32_t tcol = part == 0 ? tW : tU;
      T* dst = (part == 0 ? w + orow * K : u + orow * V);
      for (int j0 = 0; j0 < n; j0 += 32) {
        float r[32];
        tmem_ld32(tcol + la + j0, r);
        if (lane < 16) {
          if constexpr (kBf16) {
#pragma unroll
            for (int q = 0; q < 32; q += 8) {
              uint4 p;
              p.x = pack_bf16x2(r[q], r[q + 1]);
              p.y = pack_bf16x2(r[q + 2], r[q + 3]);
              p.z = pack_bf16x2(r[q + 4], r[q + 5]);
              p.w = pack_bf16x2(r[q + 6], r[q + 7]);
              *reinterpret_cast<uint4*>(dst + j0 + q) = p;
            }
          } else {
#pragma unroll
            for (int q = 0; q < 32; q += 4)
              *reinterpret_cast<float4*>(dst + j0 + q) = make_float4(r[q], r[q + 1], r[q + 2], r[q + 3]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, Ly::TMEM_COLS);
  return;

cleanup:
  // A wait ran out of time: one more bounded wait for anything in flight,
  // then release TMEM.
  mbar_wait(bar_tma, 0, &g_status_wu);
  if (pending >= 0) mbar_wait(bar_mma, (uint32_t)pending, &g_status_wu);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, Ly::TMEM_COLS);
}

template <typename T, int K, int V>
int launch(const void* k, const void* v, const float* beta, const float* A, const float* g, void* w, void* u,
           float* a_out, int B, int T_len, int H, int a_mode, cudaStream_t st) {
  using Ly = Layout<T, K, V>;
  constexpr bool bf = Ly::BF16;
  const CUtensorMapDataType dt = bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const CUtensorMapSwizzle mn_sw = bf ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  const int es = sizeof(T);
  const uint64_t rows = (uint64_t)B * T_len;
  const uint32_t box[3] = {(uint32_t)(128 / es), 1u, (uint32_t)kBT};
  CUtensorMap tk, tkk, tv, ta;
  {
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)H, rows};
    uint64_t str[2] = {(uint64_t)K * es, (uint64_t)H * K * es};
    int r = encode_tiled(&tk, dt, 3, k, dims, str, box, mn_sw);
    if (r == THM_OK) r = encode_tiled(&tkk, dt, 3, k, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (r != THM_OK) return r;
  }
  {
    uint64_t dims[3] = {(uint64_t)V, (uint64_t)H, rows};
    uint64_t str[2] = {(uint64_t)V * es, (uint64_t)H * V * es};
    int r = encode_tiled(&tv, dt, 3, v, dims, str, box, mn_sw);
    if (r != THM_OK) return r;
  }
  if (a_mode == 0) {
    uint64_t dims[3] = {(uint64_t)kBT, (uint64_t)H, rows};
    uint64_t str[2] = {(uint64_t)kBT * 4, (uint64_t)H * kBT * 4};
    uint32_t abox[3] = {32u, 1u, (uint32_t)kBT};
    int r = encode_tiled(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, A, dims, str, abox);
    if (r != THM_OK) return r;
  } else {
    ta = tk;  // unused
  }
  auto kern = recompute_w_u_kernel<T, K, V>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Ly::SMEM) != cudaSuccess)
    return THM_ERR_CUDA;
  dim3 grid(T_len / kBT, B * H);
  kern<<<grid, kThreads, Ly::SMEM, st>>>(tk, tkk, tv, ta, beta, g, static_cast<T*>(w), static_cast<T*>(u), a_out,
                                         T_len, H, a_mode);
  return check_launch();
}

template <typename T>
int dispatch(const void* k, const void* v, const float* beta, const float* A, const float* g, void* w, void* u,
             float* a_out, int B, int T_len, int H, int K, int V, int a_mode, cudaStream_t st) {
  if (K == 64 && V == 64) return launch<T, 64, 64>(k, v, beta, A, g, w, u, a_out, B, T_len, H, a_mode, st);
  if (K == 64 && V == 128) return launch<T, 64, 128>(k, v, beta, A, g, w, u, a_out, B, T_len, H, a_mode, st);
  if (K == 128 && V == 64) return launch<T, 128, 64>(k, v, beta, A, g, w, u, a_out, B, T_len, H, a_mode, st);
  if (K == 128 && V == 128) return launch<T, 128, 128>(k, v, beta, A, g, w, u, a_out, B, T_len, H, a_mode, st);
  return THM_ERR_UNSUPPORTED;
}

}  // namespace wu
}  // namespace thm

THM_STATUS_READER(thm_internal_status_wu, g_status_wu)

extern "C" int thm_recompute_w_u_fwd(const void* k, const void* v, const float* beta, const float* A,
                                     const float* g, void* w, void* u, float* A_out, int B, int T, int H, int K,
                                     int V, int dtype, int a_mode, thm_stream_t stream) {
  using namespace thm;
  if (B < 0 || T < 0 || H < 0 || K <= 0 || V <= 0 || T % 64 != 0) return THM_ERR_INVALID;
  if (dtype != THM_F32 && dtype != THM_BF16) return THM_ERR_INVALID;
  if (a_mode < -1 || a_mode > 1) return THM_ERR_INVALID;
  if ((long long)B * T * H == 0) return THM_OK;
  if (!k || !v || !beta || !g || !w || !u || (a_mode == 0 && !A)) return THM_ERR_INVALID;
  if (!(K == 64 || K == 128) || !(V == 64 || V == 128)) return THM_ERR_UNSUPPORTED;
  if (!aligned16(k) || !aligned16(v) || !aligned16(w) || !aligned16(u) || (a_mode == 0 && !aligned16(A)))
    return THM_ERR_ALIGNMENT;
  if ((long long)B * H > 65535) return THM_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == THM_BF16)
    return wu::dispatch<__nv_bfloat16>(k, v, beta, A, g, w, u, A_out, B, T, H, K, V, a_mode, st);
  return wu::dispatch<float>(k, v, beta, A, g, w, u, A_out, B, T, H, K, V, a_mode, st);
}
