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
  const bool a_only = w == nullptr;  // build_A: A (a_out) is the only output, no v tile
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
    uint32_t bytes = Ly::K_BYTES + (a_only ? 0u : (uint32_t)Ly::V_BYTES) + (fused ? Ly::KK_BYTES : Ly::AF_BYTES);
    mbar_arrive_expect_tx(bar_tma, bytes);
#pragma unroll
    for (int j = 0; j < K / kBox; ++j) {
      tma_load_3d(sm + Ly::OFF_K + j * kBT * 128, &tm_k, bar_tma, j * kBox, h, row0);
      if (!kBf16 && fused) tma_load_3d(sm + Ly::OFF_KK + j * kBT * 128, &tm_kk, bar_tma, j * kBox, h, row0);
    }
#pragma unroll
    for (int j = 0; j < V / kBox; ++j)
      if (!a_only) tma_load_3d(sm + Ly::OFF_V + j * kBT * 128, &tm_v, bar_tma, j * kBox, h, row0);
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
  } else if (!a_only && (!fused || tid >= kBT)) {
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
  if (a_only) {
    if (warp == 0) tmem_dealloc(tbase, Ly::TMEM_COLS);
    return;
  }

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
    int r = v != nullptr ? encode_tiled(&tv, dt, 3, v, dims, str, box, mn_sw) : THM_OK;
    if (v == nullptr) tv = tk;  // build_A: no v tile is loaded
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


// ===========================================================================
// Persistent warp-specialized variant: bf16 k/v/w/u, A formed in-kernel.
// One CTA per SM walks units (b, c, h), h fastest.
//   warp 0      TMA producer: k, v tiles + beta, g of a unit into a 3-stage ring
//   warp 1      tcgen05 issuer: W(i), U(i) as soon as A(i) is ready, then
//               KK^T(i+2) into the TMEM region unit i's M formation released:
//                 KK^T                  (M=64, N=64, K=K)
//                 W = (A diag(beta e^g)) k   (M=64, N=K, K=64)  TMEM lane 0
//                 U = (A diag(beta)) v       (M=64, N=V, K=64)  TMEM lane 16
//   warps 2-5 / 6-9  two math groups taking alternate units. Per unit i:
//               M from KK^T (TMEM) -> A = (I + sign M)^-1 by recursive 2x2
//               blocking (four 16x16 forward substitutions, then
//               A10 = -sign A11 M10 A00 at the 16 and then the 32 level)
//               -> the two column-scaled bf16 copies
//               of A as MMA operands; then the epilogue of the group's
//               previous unit (i-2), whose products finished meanwhile:
//               TMEM -> smem -> TMA store of w, u.
// Folding beta e^g / beta into A's columns keeps k and v raw, so the same TMA
// tiles feed KK^T (K-major) and the W/U products (MN-major B). W and U share
// TMEM columns as two M=64 accumulators at lane offsets 0 and 16.
// ===========================================================================
namespace ws {

constexpr int kThreads = 320;
constexpr int kThreadsConv = 384;  // + 2 warps forming v from the raw projection (CONV)
constexpr int kGroup = 128;
constexpr int kStages = 3;
constexpr int kConvW = 4;          // causal conv width of the fused v path
constexpr int kRawRows = 64 + kConvW - 1;  // a unit's rows plus the conv's history
constexpr int kRawBox = 72 * 128;  // 64-channel box of kRawRows rows, padded to 1024-B atoms

// CONV: the stage holds the raw projection x_v (rows t-3 .. t+63 of the unit, zero before the
// sequence start) instead of v; the conv warps overwrite rows 0..63 of it with
// v = act(conv(x_v)) before the U product reads them.
template <int K, int V, bool CONV = false>
struct Layout {
  static constexpr int KB = 64 * K * 2, VB = CONV ? (V / 64) * kRawBox : 64 * V * 2;
  static constexpr int VLBO = CONV ? kRawBox : 8192;    // stride of v's 64-column blocks
  static constexpr int STAGE = KB + VB;
  static constexpr int OFF_STAGE = 0;                    // [3] k | v
  static constexpr int OFF_GRP = kStages * STAGE;        // per math group:
  static constexpr int LDM = 68;                         //   row stride (floats) of M and A:
                                                         //   4-bank shift per row, no 8-way conflicts
  static constexpr int G_M = 0;                          //   M / T fp32 [64][68]; w staging
  static constexpr int G_A = 64 * LDM * 4;               //   A fp32 [64][68];     u staging
  static constexpr int G_AW = 2 * 64 * LDM * 4;          //   A diag(beta e^g) bf16, K-major
  static constexpr int G_AU = G_AW + 8192;               //   A diag(beta) bf16, K-major
  static constexpr int GRP = G_AU + 8192;
  static constexpr int SC = 6 * 64;                      // per stage: beta | g | beta e^g |
                                                         //   beta e^{g - g_m} | e^{g_m - g} | flag
  static constexpr int OFF_SC = OFF_GRP + 2 * GRP;
  static constexpr int OFF_BAR = OFF_SC + kStages * SC * 4;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
};

// W (lane 0) and U (lane 16) are M=64 accumulators interleaved in the same
// TMEM columns; the epilogue reads both with one 32x32b load per 32 columns.
template <int K, int V, bool CONV>
__device__ __forceinline__ void wu_epilogue(uint8_t* gb, uint32_t tbase, int grp, int sp, int lane, int mt,
                                            uint64_t* tfree_o, const CUtensorMap* tm_w, const CUtensorMap* tm_u,
                                            int hh, int row0, uint32_t bar_sync) {
  using Ly = Layout<K, V, CONV>;
  const uint32_t tW = tbase + 256 * grp + 64 + ((uint32_t)(32 * sp) << 16);
  uint8_t* ws_ = gb + Ly::G_M;
  uint8_t* us_ = gb + Ly::G_A;
  // 32x32b loads: TMEM lane 32 sp + l holds W row 16 sp + l (l < 16) or U row
  // 16 sp + l - 16 (l >= 16), 32 consecutive columns per load; each thread packs
  // its row into 16-B chunks of the row-major, 128-B-swizzled staging tiles.
  {
    const bool is_w = lane < 16;
    const int r = 16 * sp + (lane & 15);
    uint8_t* dst = is_w ? ws_ : us_;
    const int ncol = is_w ? K : V;
    constexpr int NMAX = K > V ? K : V;
#pragma unroll
    for (int c0 = 0; c0 < NMAX; c0 += 64) {
      float v[64];
      tmem_ld64(tW + c0, v);
      if (c0 < ncol) {
        uint8_t* box = dst + (c0 / 64) * 8192 + r * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint32_t ck = (uint32_t)(q ^ (r & 7));
          *reinterpret_cast<uint4*>(box + (ck << 4)) =
              make_uint4(pack_bf16x2(v[8 * q], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                         pack_bf16x2(v[8 * q + 4], v[8 * q + 5]), pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
        }
      }
    }
  }
  tc_fence_before();
  mbar_arrive(&tfree_o[grp]);
  fence_proxy_async_smem();
  named_bar_sync(bar_sync, kGroup);
  if (mt == 0) {
#pragma unroll
    for (int j = 0; j < K / 64; ++j) tma_store_3d(tm_w, ws_ + j * 8192, j * 64, hh, row0);
#pragma unroll
    for (int j = 0; j < V / 64; ++j) tma_store_3d(tm_u, us_ + j * 8192, j * 64, hh, row0);
    bulk_commit_group();
  }
}

template <int K, int V, bool CONV>
__global__ void __launch_bounds__(CONV ? kThreadsConv : kThreads, 1)
    recompute_w_u_ws_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                            const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_u,
                            const float* __restrict__ beta, const float* __restrict__ g,
                            float* __restrict__ a_out, int T_len, int H, int NT, int nunits, float sgn,
                            const float* __restrict__ conv_w, const float* __restrict__ conv_b, int silu) {
  using Ly = Layout<K, V, CONV>;
  constexpr uint32_t kIdKK = make_idesc(1u, 64, 64, 0, 0);
  constexpr uint32_t kIdW = make_idesc(1u, 64, K, 0, 1);
  constexpr uint32_t kIdU = make_idesc(1u, 64, V, 0, 1);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(sm);
  float* sSc = reinterpret_cast<float*>(sm + Ly::OFF_SC);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Ly::OFF_BAR);
  uint64_t* full = bars;          // [3] stage loaded (+ beta, g)
  uint64_t* empty = bars + 3;     // [3] stage consumed by the tensor core
  uint64_t* kfull = bars + 6;     // [2] KK^T in TMEM (per group)
  uint64_t* tfree_k = bars + 8;   // [2] KK^T region read out
  uint64_t* afull = bars + 10;    // [2] A operands in smem
  uint64_t* ofull = bars + 12;    // [2] W^T, U^T in TMEM
  uint64_t* tfree_o = bars + 14;  // [2] W/U region read out
  uint64_t* vfull = bars + 16;    // [3] CONV: v formed in the stage (one arrival per conv warp)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // units of this CTA: u_i = blockIdx.x + i * gridDim.x, i < n_local
  const int n_local = nunits > (int)blockIdx.x ? (nunits - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 33);
      mbar_init(&empty[i], 1);
      mbar_init(&vfull[i], 2);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kfull[i], 1);
      mbar_init(&tfree_k[i], kGroup);
      mbar_init(&afull[i], kGroup);
      mbar_init(&ofull[i], 1);
      mbar_init(&tfree_o[i], kGroup);
    }
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    // beta, g of unit i are loaded one unit ahead (their latency overlaps the
    // wait for the stage); row r of a unit at (row0 + r) * H + hh.
    auto gate_index = [&](int i) {
      const int u = blockIdx.x + i * gridDim.x;
      const int hh = u % H, bc = u / H, c = bc % NT, b = bc / NT;
      return (long long)(b * T_len + c * 64 + lane) * H + hh;
    };
    float nb0 = 0.f, ng0 = 0.f, nb1 = 0.f, ng1 = 0.f;
    if (n_local > 0) {
      const long long gi = gate_index(0);
      nb0 = beta[gi]; ng0 = g[gi]; nb1 = beta[gi + 32LL * H]; ng1 = g[gi + 32LL * H];
    }
    for (int i = 0; i < n_local; ++i) {
      const int u = blockIdx.x + i * gridDim.x;
      const int st = i % kStages;
      const float bv0 = nb0, gv0 = ng0, bv1 = nb1, gv1 = ng1;
      if (i + 1 < n_local) {
        const long long gi = gate_index(i + 1);
        nb0 = beta[gi]; ng0 = g[gi]; nb1 = beta[gi + 32LL * H]; ng1 = g[gi + 32LL * H];
      }
      if (i >= kStages) {
        ok = __all_sync(0xffffffffu, mbar_wait(&empty[st], ((i / kStages) & 1) ^ 1, &g_status_wu));
        if (!ok) break;
      }
      const int hh = u % H, bc = u / H, c = bc % NT, b = bc / NT;
      const int row0 = b * T_len + c * 64;
      float* sc = sSc + st * Ly::SC;
      if (lane == 0) {
        uint8_t* stg = sm + Ly::OFF_STAGE + st * Ly::STAGE;
        mbar_arrive_expect_tx(&full[st], CONV ? Ly::KB + (V / 64) * kRawRows * 128 : Ly::STAGE);
#pragma unroll
        for (int j = 0; j < K / 64; ++j) tma_load_3d(stg + j * 8192, &tm_k, &full[st], j * 64, hh, row0);
#pragma unroll
        for (int j = 0; j < V / 64; ++j) {
          if constexpr (CONV)  // x_v [B, T, H, V]: rows c*64-3 .. c*64+63 of sequence b
            tma_load_4d(stg + Ly::KB + j * kRawBox, &tm_v, &full[st], j * 64, hh, c * 64 - (kConvW - 1), b);
          else
            tma_load_3d(stg + Ly::KB + j * 8192, &tm_v, &full[st], j * 64, hh, row0);
        }
        if (i + 1 < n_local) {
          // the next unit's tiles into L2 now: its load is issued once a stage frees
          // (a unit later) and then comes from L2 instead of HBM
          const int un = u + gridDim.x;
          const int hn = un % H, bn = un / H;
          const int rn = (bn / NT) * T_len + (bn % NT) * 64;
#pragma unroll
          for (int j = 0; j < K / 64; ++j) tma_prefetch_l2_3d(&tm_k, j * 64, hn, rn);
#pragma unroll
          for (int j = 0; j < V / 64; ++j) {
            if constexpr (CONV)
              tma_prefetch_l2_4d(&tm_v, j * 64, hn, (bn % NT) * 64 - (kConvW - 1), bn / NT);
            else
              tma_prefetch_l2_3d(&tm_v, j * 64, hn, rn);
          }
        }
      }
      // Decay e^{g_r - g_c} = e^{g_r - g_m} e^{g_m - g_c} about the middle g_m of the
      // chunk's gate range (each factor at most e^{range/2}; ranges over 120 keep one
      // exponential per entry, flag 0).
      float mn = fminf(gv0, gv1), mx = fmaxf(gv0, gv1);
#pragma unroll
      for (int m = 16; m >= 1; m >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, m));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m));
      }
      const float gm = 0.5f * (mn + mx);
      sc[lane] = bv0;
      sc[32 + lane] = bv1;
      sc[64 + lane] = gv0;
      sc[96 + lane] = gv1;
      sc[128 + lane] = bv0 * __expf(gv0);
      sc[160 + lane] = bv1 * __expf(gv1);
      sc[192 + lane] = bv0 * __expf(gv0 - gm);
      sc[224 + lane] = bv1 * __expf(gv1 - gm);
      sc[256 + lane] = __expf(gm - gv0);
      sc[288 + lane] = __expf(gm - gv1);
      if (lane == 0) sc[320] = (mx - mn <= 120.f) ? 1.f : 0.f;
      mbar_arrive(&full[st]);
    }
  } else if (warp == 1) {
    // ---------------- tcgen05 issuer ----------------
    // Two independent streams, issued in whatever order their inputs arrive:
    //   KK^T(i) needs stage i loaded and unit i-2's M formation done;
    //   W/U(i)  needs A(i) written and unit i-2's W/U read out.
    if (lane == 0) {
      int next_kk = 0, next_wu = 0;
      uint64_t t_last = globaltimer_ns();
      while (next_wu < n_local) {
        bool did = false;
        if (next_kk < n_local) {
          const int i = next_kk, st = i % kStages, gi = i & 1;
          if (mbar_test(&full[st], (i / kStages) & 1) &&
              (i < 2 || mbar_test(&tfree_k[gi], ((i >> 1) & 1) ^ 1))) {
            tc_fence_after();
            const uint32_t sk = sbase + Ly::OFF_STAGE + st * Ly::STAGE;
#pragma unroll
            for (int q = 0; q < K / 16; ++q) {
              const uint64_t d = make_sdesc(sk + (q / 4) * 8192 + (q % 4) * 32, 16, 1024);
              mma_bf16_ss(tbase + 256 * gi, d, d, kIdKK, q > 0);
            }
            mma_commit(&kfull[gi]);
            ++next_kk;
            did = true;
          }
        }
        if (next_wu < next_kk) {
          const int i = next_wu, st = i % kStages, gi = i & 1;
          const uint32_t ph = (i >> 1) & 1;
          if (mbar_test(&afull[gi], ph) && (i < 2 || mbar_test(&tfree_o[gi], ph ^ 1)) &&
              (!CONV || mbar_test(&vfull[st], (i / kStages) & 1))) {
            tc_fence_after();
            const uint32_t sk = sbase + Ly::OFF_STAGE + st * Ly::STAGE;
            const uint32_t sv = sk + Ly::KB;
            const uint32_t grp = sbase + Ly::OFF_GRP + gi * Ly::GRP;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint64_t aw = make_sdesc(grp + Ly::G_AW + q * 32, 16, 1024);
              const uint64_t au = make_sdesc(grp + Ly::G_AU + q * 32, 16, 1024);
              // W = A_w k at TMEM lane 0, U = A_u v at lane 16 (interleaved M=64 accumulators)
              mma_bf16_ss(tbase + 256 * gi + 64, aw, make_sdesc(sk + q * 2048, 8192, 1024), kIdW, q > 0);
              mma_bf16_ss(tbase + 256 * gi + 64 + (16u << 16), au, make_sdesc(sv + q * 2048, Ly::VLBO, 1024), kIdU,
                          q > 0);
            }
            mma_commit(&ofull[gi]);
            mma_commit(&empty[st]);
            ++next_wu;
            did = true;
          }
        }
        const uint64_t now = globaltimer_ns();
        if (did) {
          t_last = now;
        } else if (now - t_last > kWaitLimitNs) {
          record_status(&g_status_wu, THM_ERR_TIMEOUT);
          ok = false;
          break;
        } else {
          // back off: a tight poll would take issue slots from the math warp
          // sharing this SM sub-partition
          __nanosleep(64);
        }
      }
    }
  } else if (CONV && warp >= kThreads / 32) {
    // ---------------- conv warps (CONV) ----------------
    // v = act(bias + sum_k w[k] x[t-3+k]) for one channel pair per thread, in place: row t of
    // the stage's raw tile (which held x[t-3], already in this thread's window) receives
    // v[t]. Same arithmetic as the causal_conv1d kernel's bf16 path (packed fp32x2 fmas in
    // tap order, silu as h + h tanh(h)), so v equals that kernel's output bit for bit.
    const int ct = tid - kThreads;  // channel pair 2 ct, 2 ct + 1 of the head
    const bool active = ct < V / 2;
    const uint32_t cb = (uint32_t)(ct & 31) * 4;  // byte of the pair in a 128-B row
    for (int i = 0; i < n_local && ok; ++i) {
      const int u = blockIdx.x + i * gridDim.x;
      const int st = i % kStages;
      const int hh = u % H;
      float2 wk[kConvW], bias2 = make_float2(0.f, 0.f);
      if (active) {
        const long long ch = (long long)hh * V + 2 * ct;
        bias2 = make_float2(__ldg(conv_b + ch), __ldg(conv_b + ch + 1));
#pragma unroll
        for (int k = 0; k < kConvW; ++k) wk[k] = make_float2(__ldg(conv_w + ch * kConvW + k), __ldg(conv_w + (ch + 1) * kConvW + k));
      }
      ok = __all_sync(0xffffffffu, mbar_wait(&full[st], (i / kStages) & 1, &g_status_wu));
      if (!ok) break;
      if (active) {
        uint8_t* box = sm + Ly::OFF_STAGE + st * Ly::STAGE + Ly::KB + (ct >> 5) * kRawBox;
        auto at = [&](int r) -> uint32_t* {
          return reinterpret_cast<uint32_t*>(box + r * 128 + (((cb >> 4) ^ (uint32_t)(r & 7)) << 4) + (cb & 15));
        };
        auto ld2 = [&](int r) {
          const uint32_t x = *at(r);
          return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x));
        };
        // Rows in batches of 8: the batch's raw rows t0+3 .. t0+10 are read before rows
        // t0 .. t0+7 are overwritten, so loads, the 8 independent outputs and the stores
        // pipeline instead of each step waiting on the previous one's store.
        constexpr int kBatch = 8;
        float2 xw[kConvW - 1 + kBatch];
#pragma unroll
        for (int r = 0; r < kConvW - 1; ++r) xw[r] = ld2(r);
#pragma unroll 1
        for (int t0 = 0; t0 < 64; t0 += kBatch) {
#pragma unroll
          for (int r = 0; r < kBatch; ++r) xw[kConvW - 1 + r] = ld2(t0 + kConvW - 1 + r);
          uint32_t outp[kBatch];
#pragma unroll
          for (int r = 0; r < kBatch; ++r) {
            float2 acc = bias2;
#pragma unroll
            for (int k = 0; k < kConvW; ++k) acc = __ffma2_rn(xw[r + k], wk[k], acc);
            if (silu) {
              const float2 h = __fmul2_rn(make_float2(0.5f, 0.5f), acc);
              float t0h, t1h;
              asm("tanh.approx.f32 %0, %1;" : "=f"(t0h) : "f"(h.x));
              asm("tanh.approx.f32 %0, %1;" : "=f"(t1h) : "f"(h.y));
              acc = __ffma2_rn(h, make_float2(t0h, t1h), h);
            }
            outp[r] = pack_bf16x2(acc.x, acc.y);
          }
#pragma unroll
          for (int r = 0; r < kBatch; ++r) *at(t0 + r) = outp[r];
#pragma unroll
          for (int r = 0; r < kConvW - 1; ++r) xw[r] = xw[kBatch + r];
        }
      }
      fence_proxy_async_smem();  // the tensor core reads v through the async proxy
      __syncwarp();
      if (lane == 0) mbar_arrive(&vfull[st]);
    }
  } else {
    // ---------------- math groups ----------------
    const int grp = (warp - 2) >> 2;  // 0: warps 2-5, 1: warps 6-9
    const int mt = tid - 64 - grp * kGroup;
    const int sp = warp & 3;          // TMEM subpartition of this warp
    const uint32_t lane_base = (uint32_t)(32 * sp) << 16;
    const uint32_t bar_sync = 1 + grp, bar_vote = 3 + grp;
    uint8_t* gb = sm + Ly::OFF_GRP + grp * Ly::GRP;
    float(*sM)[Ly::LDM] = reinterpret_cast<float(*)[Ly::LDM]>(gb + Ly::G_M);
    float(*sA)[Ly::LDM] = reinterpret_cast<float(*)[Ly::LDM]>(gb + Ly::G_A);
    int prev_hh = 0, prev_row0 = 0;
    bool has_prev = false;
    {
      // Rows 0..31, columns 32..63 of A are zero and never rewritten: zero them in
      // both bf16 operand tiles once (made visible to the tensor core by the fence
      // before the first afull arrival).
      const int r = mt >> 2, ck = 4 + (mt & 3);
      const uint32_t off = (uint32_t)r * 128u + ((uint32_t)(ck ^ (r & 7)) << 4);
      *reinterpret_cast<uint4*>(gb + Ly::G_AW + off) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(gb + Ly::G_AU + off) = make_uint4(0, 0, 0, 0);
    }
    // Converts 8 consecutive entries of a row of A (fp32, columns c0..c0+7, already
    // masked) into the two column-scaled bf16 MMA operands (and the optional fp32 A).
    auto put_a8 = [&](const float* a, int t, int c0, const float* sc, int hh, int row0) {
      const float* fk = sc + 128 + c0;
      const float* fb = sc + c0;
      uint32_t w4[4], u4[4];
#pragma unroll
      for (int z = 0; z < 4; ++z) {  // packed fp32x2 products (same rounding as scalar)
        const float2 a2 = make_float2(a[2 * z], a[2 * z + 1]);
        const float2 pw2 = __fmul2_rn(a2, make_float2(fk[2 * z], fk[2 * z + 1]));
        const float2 pu2 = __fmul2_rn(a2, make_float2(fb[2 * z], fb[2 * z + 1]));
        w4[z] = pack_bf16x2(pw2.x, pw2.y);
        u4[z] = pack_bf16x2(pu2.x, pu2.y);
      }
      const uint4 pw = make_uint4(w4[0], w4[1], w4[2], w4[3]), pu = make_uint4(u4[0], u4[1], u4[2], u4[3]);
      *reinterpret_cast<uint4*>(gb + Ly::G_AW + sw128_offset(t, c0, 64, 2)) = pw;
      *reinterpret_cast<uint4*>(gb + Ly::G_AU + sw128_offset(t, c0, 64, 2)) = pu;
      if (a_out != nullptr) {
        float* dst = a_out + ((long long)(row0 + t) * H + hh) * 64 + c0;
        *reinterpret_cast<float4*>(dst) = make_float4(a[0], a[1], a[2], a[3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(a[4], a[5], a[6], a[7]);
      }
    };
    // The same for 4 consecutive entries (columns c0..c0+3, c0 % 4 == 0).
    auto put_a4 = [&](const float* a, int t, int c0, const float* sc, int hh, int row0) {
      const float* fk = sc + 128 + c0;
      const float* fb = sc + c0;
      const float2 a01 = make_float2(a[0], a[1]), a23 = make_float2(a[2], a[3]);
      const float2 w01 = __fmul2_rn(a01, make_float2(fk[0], fk[1])), w23 = __fmul2_rn(a23, make_float2(fk[2], fk[3]));
      const float2 u01 = __fmul2_rn(a01, make_float2(fb[0], fb[1])), u23 = __fmul2_rn(a23, make_float2(fb[2], fb[3]));
      const uint32_t off = sw128_offset(t, c0, 64, 2);
      *reinterpret_cast<uint2*>(gb + Ly::G_AW + off) = make_uint2(pack_bf16x2(w01.x, w01.y), pack_bf16x2(w23.x, w23.y));
      *reinterpret_cast<uint2*>(gb + Ly::G_AU + off) = make_uint2(pack_bf16x2(u01.x, u01.y), pack_bf16x2(u23.x, u23.y));
      if (a_out != nullptr)
        *reinterpret_cast<float4*>(a_out + ((long long)(row0 + t) * H + hh) * 64 + c0) = make_float4(a[0], a[1], a[2], a[3]);
    };
    for (int i = grp; i < n_local; i += 2) {
      const int u = blockIdx.x + i * gridDim.x;
      const int st = i % kStages;
      const uint32_t ph = (i >> 1) & 1;
      const int hh = u % H, bc = u / H, c = bc % NT, b = bc / NT;
      const int row0 = b * T_len + c * 64;
      const float* sc = sSc + st * Ly::SC;
      ok = mbar_wait(&full[st], (i / kStages) & 1, &g_status_wu) && mbar_wait(&kfull[grp], ph, &g_status_wu);
      if (!named_bar_and(bar_vote, kGroup, ok)) { ok = false; break; }
      tc_fence_after();
      {
        // M_rc = beta_r (k_r.k_c) e^{g_r - g_c}, c < r
        float kv[32];
        tmem_ld_16x256b_x8(tbase + 256 * grp + lane_base, kv);
        tc_fence_before();
        mbar_arrive(&tfree_k[grp]);
        const int r0 = 16 * sp + (lane >> 2), r1 = r0 + 8;
        const float b0 = sc[r0], b1 = sc[r1], g0 = sc[64 + r0], g1 = sc[64 + r1];
        const float fa0 = sc[192 + r0], fa1 = sc[192 + r1];
        const bool factored = sc[320] != 0.f;  // uniform
        // Only the strictly lower triangle of M is ever read (the solve below and
        // T = M10 A00): this warp's rows 16sp..16sp+15 need column groups j <= 2sp+1.
        float2 m0[8], m1[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (j > 2 * sp + 1) break;  // warp-uniform
          const int cc = 8 * j + 2 * (lane & 3);
          if (factored) {
            const float2 fb = make_float2(sc[256 + cc], sc[256 + cc + 1]);
            // (fa kv) fb, left to right as the scalar form, as packed fp32x2
            const float2 p0 = __fmul2_rn(__fmul2_rn(make_float2(fa0, fa0), make_float2(kv[4 * j], kv[4 * j + 1])), fb);
            const float2 p1 =
                __fmul2_rn(__fmul2_rn(make_float2(fa1, fa1), make_float2(kv[4 * j + 2], kv[4 * j + 3])), fb);
            m0[j].x = (cc < r0) ? p0.x : 0.f;
            m0[j].y = (cc + 1 < r0) ? p0.y : 0.f;
            m1[j].x = (cc < r1) ? p1.x : 0.f;
            m1[j].y = (cc + 1 < r1) ? p1.y : 0.f;
          } else {
            const float gc0 = sc[64 + cc], gc1 = sc[64 + cc + 1];
            m0[j].x = (cc < r0) ? b0 * kv[4 * j] * __expf(g0 - gc0) : 0.f;
            m0[j].y = (cc + 1 < r0) ? b0 * kv[4 * j + 1] * __expf(g0 - gc1) : 0.f;
            m1[j].x = (cc < r1) ? b1 * kv[4 * j + 2] * __expf(g1 - gc0) : 0.f;
            m1[j].y = (cc + 1 < r1) ? b1 * kv[4 * j + 3] * __expf(g1 - gc1) : 0.f;
          }
        }
        // the previous unit's w/u tiles (staged in sM / sA) have left shared memory:
        // waited only now, so the TMA store drains while KK^T is read and scaled
        if (mt == 0) bulk_wait_group_read0();
        named_bar_sync(bar_sync, kGroup);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (j > 2 * sp + 1) break;
          const int cc = 8 * j + 2 * (lane & 3);
          *reinterpret_cast<float2*>(&sM[r0][cc]) = m0[j];
          *reinterpret_cast<float2*>(&sM[r1][cc]) = m1[j];
        }
      }
      named_bar_sync(bar_sync, kGroup);
      // (1a) four diagonal 16x16 blocks by column-parallel forward substitution
      if (mt < 64) {
        const int blk = mt >> 4, j = mt & 15, base = 16 * blk;
        float x[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) x[q] = 0.f;
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          float2 s01 = make_float2(0.f, 0.f), s23 = make_float2(0.f, 0.f);
#pragma unroll
          for (int m = 0; m < r; m += 4) {
            const float4 mv = *reinterpret_cast<const float4*>(&sM[base + r][base + m]);
            s01 = __ffma2_rn(make_float2(mv.x, mv.y), make_float2(x[m], x[m + 1]), s01);
            s23 = __ffma2_rn(make_float2(mv.z, mv.w), make_float2(x[m + 2], x[m + 3]), s23);
          }
          x[r] = ((r == j) ? 1.f : 0.f) - sgn * ((s01.x + s01.y) + (s23.x + s23.y));
        }
        // Only the lower-triangular blocks of sA are ever written; readers
        // below never touch the (unwritten) upper-right blocks.
#pragma unroll
        for (int r = 0; r < 16; ++r) sA[base + r][base + j] = x[r];
      }
      named_bar_sync(bar_sync, kGroup);
      // (1b) inside each 32x32 block: A_10 = -sign A_11 (M_10 A_00) on 16x16 blocks.
      //      128 threads = 2 blocks x 16 rows x 4 column groups of 4.
      {
        const int p = mt >> 6, r = (mt >> 2) & 15, c4 = (mt & 3) * 4, base = 32 * p;
        float2 t01 = make_float2(0.f, 0.f), t23 = make_float2(0.f, 0.f);
#pragma unroll
        for (int m = 0; m < 16; ++m) {
          const float mv = sM[base + 16 + r][base + m];
          const float4 a = *reinterpret_cast<const float4*>(&sA[base + m][base + c4]);
          t01 = __ffma2_rn(make_float2(mv, mv), make_float2(a.x, a.y), t01);
          t23 = __ffma2_rn(make_float2(mv, mv), make_float2(a.z, a.w), t23);
        }
        const float t4[4] = {t01.x, t01.y, t23.x, t23.y};
        named_bar_sync(bar_sync, kGroup);  // M_00 corners no longer read
        *reinterpret_cast<float4*>(&sM[base + r][base + c4]) = make_float4(t4[0], t4[1], t4[2], t4[3]);
        named_bar_sync(bar_sync, kGroup);
        float2 a01 = make_float2(0.f, 0.f), a23 = make_float2(0.f, 0.f);
#pragma unroll
        for (int m = 0; m < 16; ++m) {
          const float av = sA[base + 16 + r][base + 16 + m];
          const float4 t = *reinterpret_cast<const float4*>(&sM[base + m][base + c4]);
          a01 = __ffma2_rn(make_float2(av, av), make_float2(t.x, t.y), a01);
          a23 = __ffma2_rn(make_float2(av, av), make_float2(t.z, t.w), a23);
        }
        const float a4[4] = {a01.x, a01.y, a23.x, a23.y};
        *reinterpret_cast<float4*>(&sA[base + 16 + r][base + c4]) =
            make_float4(-sgn * a4[0], -sgn * a4[1], -sgn * a4[2], -sgn * a4[3]);
      }
      // the previous unit's W/U products have consumed the A operand tiles
      ok = !has_prev || mbar_wait(&ofull[grp], ph ^ 1, &g_status_wu);
      if (!named_bar_and(bar_vote, kGroup, ok)) { ok = false; break; }
      // (2) T = M10 A00, written into the A10 slot of sA (A10 itself goes straight to
      //     the operand tiles, so the slot is free and nothing in this phase reads
      //     it: no barrier between the products and the write). Alongside: the diagonal
      //     32-blocks A00, A11 are final, so their operand entries are written now
      //     (thread: block mt/64, row (mt/2)%32, 16 columns).
      // products: thread = rows 2 rp, 2 rp + 1 x columns tc .. tc + 3 (register-blocked:
      // one float4 of each M / A row serves four m)
      const int rp = mt >> 3, tc = (mt & 7) * 4;
      {
        const int blk = mt >> 6, rr = (mt >> 1) & 31, cb0 = (mt & 1) * 16;
        const int t = 32 * blk + rr;
#pragma unroll
        for (int q = 0; q < 16; q += 8) {
          float a[8];
          *reinterpret_cast<float4*>(a) = *reinterpret_cast<const float4*>(&sA[t][32 * blk + cb0 + q]);
          *reinterpret_cast<float4*>(a + 4) = *reinterpret_cast<const float4*>(&sA[t][32 * blk + cb0 + q + 4]);
#pragma unroll
          for (int e = 0; e < 8; ++e) a[e] = (cb0 + q + e <= rr) ? a[e] : 0.f;  // upper triangle unwritten
          put_a8(a, t, 32 * blk + cb0 + q, sc, hh, row0);
        }
        if (blk == 0 && a_out != nullptr) {
          // the zero block (rows 0..31, columns 32..63) of the fp32 A
          float* dst = a_out + ((long long)(row0 + t) * H + hh) * 64 + 32 + cb0;
#pragma unroll
          for (int q = 0; q < 16; q += 4) *reinterpret_cast<float4*>(dst + q) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      {
        // packed fp32x2 FMAs (each lane an fmaf, summed over m in order as before)
        float2 t0a = make_float2(0.f, 0.f), t0b = t0a, t1a = t0a, t1b = t0a;
        // A00 is lower triangular: rows m < 16 only touch columns < 16
#pragma unroll 2
        for (int m4 = (tc >= 16 ? 16 : 0); m4 < 32; m4 += 4) {
          const float4 ma = *reinterpret_cast<const float4*>(&sM[32 + 2 * rp][m4]);
          const float4 mb = *reinterpret_cast<const float4*>(&sM[33 + 2 * rp][m4]);
          const float mav[4] = {ma.x, ma.y, ma.z, ma.w}, mbv[4] = {mb.x, mb.y, mb.z, mb.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float4 a = *reinterpret_cast<const float4*>(&sA[m4 + e][tc]);
            const float2 alo = make_float2(a.x, a.y), ahi = make_float2(a.z, a.w);
            t0a = __ffma2_rn(make_float2(mav[e], mav[e]), alo, t0a);
            t0b = __ffma2_rn(make_float2(mav[e], mav[e]), ahi, t0b);
            t1a = __ffma2_rn(make_float2(mbv[e], mbv[e]), alo, t1a);
            t1b = __ffma2_rn(make_float2(mbv[e], mbv[e]), ahi, t1b);
          }
        }
        *reinterpret_cast<float4*>(&sA[32 + 2 * rp][tc]) = make_float4(t0a.x, t0a.y, t0b.x, t0b.y);
        *reinterpret_cast<float4*>(&sA[33 + 2 * rp][tc]) = make_float4(t1a.x, t1a.y, t1b.x, t1b.y);
      }
      named_bar_sync(bar_sync, kGroup);
      // (3) A10 = -sign A11 T
      {
        float2 a0a = make_float2(0.f, 0.f), a0b = a0a, a1a = a0a, a1b = a0a;
        // A11 is lower triangular: rows 2 rp, 2 rp + 1 < 16 only have columns m < 16
#pragma unroll 2
        for (int m4 = 0; m4 < (rp < 8 ? 16 : 32); m4 += 4) {
          const float4 xa = *reinterpret_cast<const float4*>(&sA[32 + 2 * rp][32 + m4]);
          const float4 xb = *reinterpret_cast<const float4*>(&sA[33 + 2 * rp][32 + m4]);
          const float xav[4] = {xa.x, xa.y, xa.z, xa.w}, xbv[4] = {xb.x, xb.y, xb.z, xb.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float4 tt = *reinterpret_cast<const float4*>(&sA[32 + m4 + e][tc]);  // T row m
            const float2 tlo = make_float2(tt.x, tt.y), thi = make_float2(tt.z, tt.w);
            a0a = __ffma2_rn(make_float2(xav[e], xav[e]), tlo, a0a);
            a0b = __ffma2_rn(make_float2(xav[e], xav[e]), thi, a0b);
            a1a = __ffma2_rn(make_float2(xbv[e], xbv[e]), tlo, a1a);
            a1b = __ffma2_rn(make_float2(xbv[e], xbv[e]), thi, a1b);
          }
        }
        // A10 is final here: straight into the operand tiles (no shared-memory copy)
        const float r0[4] = {-sgn * a0a.x, -sgn * a0a.y, -sgn * a0b.x, -sgn * a0b.y};
        const float r1[4] = {-sgn * a1a.x, -sgn * a1a.y, -sgn * a1b.x, -sgn * a1b.y};
        put_a4(r0, 32 + 2 * rp, tc, sc, hh, row0);
        put_a4(r1, 33 + 2 * rp, tc, sc, hh, row0);
      }
      fence_proxy_async_smem();
      mbar_arrive(&afull[grp]);
      named_bar_sync(bar_sync, kGroup);  // sA / sM reads done before they become staging
      if (has_prev) {
        tc_fence_after();
        wu_epilogue<K, V, CONV>(gb, tbase, grp, sp, lane, mt, tfree_o, &tm_w, &tm_u, prev_hh, prev_row0, bar_sync);
      }
      has_prev = true;
      prev_hh = hh;
      prev_row0 = row0;
    }
    if (ok && has_prev) {
      // epilogue of this group's last unit
      const int last = grp + 2 * ((n_local - 1 - grp) / 2);
      ok = mbar_wait(&ofull[grp], (last >> 1) & 1, &g_status_wu);
      if (named_bar_and(bar_vote, kGroup, ok)) {
        tc_fence_after();
        if (mt == 0) bulk_wait_group_read0();
        named_bar_sync(bar_sync, kGroup);
        wu_epilogue<K, V, CONV>(gb, tbase, grp, sp, lane, mt, tfree_o, &tm_w, &tm_u, prev_hh, prev_row0, bar_sync);
      } else {
        ok = false;
      }
    }
    if (mt == 0) bulk_wait_group0();
  }

  if (!ok) record_status(&g_status_wu, THM_ERR_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 512);
}

// conv_w == nullptr: v is given. Else v is the raw projection x_v [B, T, H, V] and the
// kernel forms v = act(causal_conv1d(x_v, conv_w, conv_b)) (width kConvW) itself.
template <int K, int V, bool CONV>
int launch(const void* k, const void* v, const float* beta, const float* g, void* w, void* u, float* a_out, int B,
           int T_len, int H, int a_mode, const float* conv_w, const float* conv_b, int silu, cudaStream_t st) {
  using Ly = Layout<K, V, CONV>;
  const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int NT = T_len / 64;
  const uint64_t rows = (uint64_t)B * T_len;
  const uint32_t box[3] = {64u, 1u, 64u};
  CUtensorMap tk, tv, tw, tu;
  {
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)H, rows};
    uint64_t str[2] = {(uint64_t)K * 2, (uint64_t)H * K * 2};
    int r = encode_tiled(&tk, dt, 3, k, dims, str, box);
    if (r == THM_OK) r = encode_tiled(&tw, dt, 3, w, dims, str, box);
    if (r != THM_OK) return r;
  }
  {
    uint64_t dims[3] = {(uint64_t)V, (uint64_t)H, rows};
    uint64_t str[2] = {(uint64_t)V * 2, (uint64_t)H * V * 2};
    int r = encode_tiled(&tu, dt, 3, u, dims, str, box);
    if (r == THM_OK) {
      if constexpr (CONV) {
        const uint64_t dims4[4] = {(uint64_t)V, (uint64_t)H, (uint64_t)T_len, (uint64_t)B};
        const uint64_t str4[3] = {(uint64_t)V * 2, (uint64_t)H * V * 2, (uint64_t)T_len * H * V * 2};
        const uint32_t box4[4] = {64u, 1u, (uint32_t)kRawRows, 1u};
        r = encode_tiled(&tv, dt, 4, v, dims4, str4, box4);
      } else {
        r = encode_tiled(&tv, dt, 3, v, dims, str, box);
      }
    }
    if (r != THM_OK) return r;
  }
  auto kern = recompute_w_u_ws_kernel<K, V, CONV>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Ly::SMEM) != cudaSuccess)
    return THM_ERR_CUDA;
  const int nunits = B * NT * H;
  const int grid = nunits < sm_count() ? nunits : sm_count();
  kern<<<grid, CONV ? kThreadsConv : kThreads, Ly::SMEM, st>>>(tk, tv, tw, tu, beta, g, a_out, T_len, H, NT, nunits,
                                                              a_mode > 0 ? 1.0f : -1.0f, conv_w, conv_b, silu);
  return check_launch();
}

}  // namespace ws
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
  if (dtype == THM_BF16 && a_mode != 0) {
    // In-kernel A with bf16 operands: the persistent warp-specialized kernel.
    if (K == 64)
      return V == 64 ? wu::ws::launch<64, 64, false>(k, v, beta, g, w, u, A_out, B, T, H, a_mode, nullptr, nullptr, 0, st)
                     : wu::ws::launch<64, 128, false>(k, v, beta, g, w, u, A_out, B, T, H, a_mode, nullptr, nullptr, 0, st);
    return V == 64 ? wu::ws::launch<128, 64, false>(k, v, beta, g, w, u, A_out, B, T, H, a_mode, nullptr, nullptr, 0, st)
                   : wu::ws::launch<128, 128, false>(k, v, beta, g, w, u, A_out, B, T, H, a_mode, nullptr, nullptr, 0, st);
  }
  if (dtype == THM_BF16)
    return wu::dispatch<__nv_bfloat16>(k, v, beta, A, g, w, u, A_out, B, T, H, K, V, a_mode, st);
  return wu::dispatch<float>(k, v, beta, A, g, w, u, A_out, B, T, H, K, V, a_mode, st);
}

extern "C" int thm_recompute_w_u_conv_fwd(const void* k, const void* xv, const float* conv_w, const float* conv_b,
                                          const float* beta, const float* g, void* w, void* u, float* A_out, int B,
                                          int T, int H, int K, int V, int conv_width, int activation, int a_mode,
                                          thm_stream_t stream) {
  using namespace thm;
  if (B < 0 || T < 0 || H < 0 || K <= 0 || V <= 0 || T % 64 != 0) return THM_ERR_INVALID;
  if (a_mode != 1 && a_mode != -1) return THM_ERR_INVALID;
  if (activation != THM_ACT_NONE && activation != THM_ACT_SILU) return THM_ERR_INVALID;
  if ((long long)B * T * H == 0) return THM_OK;
  if (!k || !xv || !conv_w || !conv_b || !beta || !g || !w || !u) return THM_ERR_INVALID;
  if (!(K == 64 || K == 128) || !(V == 64 || V == 128) || conv_width != wu::ws::kConvW) return THM_ERR_UNSUPPORTED;
  if (!aligned16(k) || !aligned16(xv) || !aligned16(w) || !aligned16(u) || (A_out && !aligned16(A_out)))
    return THM_ERR_ALIGNMENT;
  if ((long long)B * H > 65535) return THM_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int silu = activation == THM_ACT_SILU;
  if (K == 64)
    return V == 64 ? wu::ws::launch<64, 64, true>(k, xv, beta, g, w, u, A_out, B, T, H, a_mode, conv_w, conv_b, silu, st)
                   : wu::ws::launch<64, 128, true>(k, xv, beta, g, w, u, A_out, B, T, H, a_mode, conv_w, conv_b, silu, st);
  return V == 64 ? wu::ws::launch<128, 64, true>(k, xv, beta, g, w, u, A_out, B, T, H, a_mode, conv_w, conv_b, silu, st)
                 : wu::ws::launch<128, 128, true>(k, xv, beta, g, w, u, A_out, B, T, H, a_mode, conv_w, conv_b, silu, st);
}

extern "C" int thm_build_A_fwd(const void* k, const float* beta, const float* g, float* A, int B, int T, int H,
                               int K, int dtype, int sign, thm_stream_t stream) {
  using namespace thm;
  if (B < 0 || T < 0 || H < 0 || K <= 0 || T % 64 != 0) return THM_ERR_INVALID;
  if (dtype != THM_F32 && dtype != THM_BF16) return THM_ERR_INVALID;
  if (sign != -1 && sign != 1) return THM_ERR_INVALID;
  if ((long long)B * T * H == 0) return THM_OK;
  if (!k || !beta || !g || !A) return THM_ERR_INVALID;
  if (!(K == 64 || K == 128)) return THM_ERR_UNSUPPORTED;
  if (!aligned16(k)) return THM_ERR_ALIGNMENT;
  if ((long long)B * H > 65535) return THM_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // The one-CTA-per-chunk kernel with no v tile and no w, u outputs.
  if (dtype == THM_BF16)
    return K == 64 ? wu::launch<__nv_bfloat16, 64, 64>(k, nullptr, beta, nullptr, g, nullptr, nullptr, A, B, T, H, sign, st)
                   : wu::launch<__nv_bfloat16, 128, 64>(k, nullptr, beta, nullptr, g, nullptr, nullptr, A, B, T, H, sign, st);
  return K == 64 ? wu::launch<float, 64, 64>(k, nullptr, beta, nullptr, g, nullptr, nullptr, A, B, T, H, sign, st)
                 : wu::launch<float, 128, 64>(k, nullptr, beta, nullptr, g, nullptr, nullptr, A, B, T, H, sign, st);
}
