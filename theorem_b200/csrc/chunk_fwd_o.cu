// chunk_fwd_o.cu -- gated-DeltaNet chunkwise output on tcgen05 tensor cores.
//
// Replaces kernels/chunk_fwd_o/kernel.py:52-136 (_chunk_fwd_o_kernel) and its
// launcher :146-212. Three kernels: fp32 activations (the reference contract)
// take the one-CTA-per-tile kernel below; bf16 activations take a persistent
// warp-specialized kernel, with a bf16 h (ws::) or an fp32 h (ws32::).
//
// fp32 kernel, per (b, h, chunk c, 64-wide V tile):
//
//   S = q k^T                                (M=64, N=64,  K=K)  tensor core
//   G = q h[c]                               (M=64, N=VT,  K=K)  tensor core, tf32
//   P = tril_{s<=t}(S * exp(g_t - g_s))      registers (TMEM -> regs -> smem)
//   L = P v                                  (M=64, N=VT,  K=64) tensor core
//   o = scale * (L + exp(g_t) * G)           registers (TMEM -> regs -> HBM)
//
// This equals the reference's scale*(tril((q e^g) k^T) (v e^-g) + (q e^g) h)
// (kernels/chunk_fwd_o/reference.py:103-140); the decay is formed on the
// masked 64x64 tile so no exp(-g) factor can overflow, and exp(g_t) is applied
// to G's rows in the epilogue instead of to q.
//
// Data movement: q, k, v tiles and the fp32 state tile h[c][:, v-tile] arrive
// by TMA on one mbarrier, already in UMMA canonical layouts: 128-B swizzle
// (16-B chunks) for K-major tiles, 128-B swizzle with 32-B atoms for the
// MN-major tf32 tiles (h, v); the accumulators live in TMEM (G: VT columns,
// S then L: 64 columns). All products run in kind::tf32, S and L as 3xTF32
// (x = hi + lo, hi = tf32(x): hi*hi + hi*lo + lo*hi), which keeps them at
// fp32 accuracy; the lo tiles of q and k are reused for lo(P) once S is done.
#include <cuda_bf16.h>

#include "host_util.h"
#include "sm100.cuh"

THM_DEFINE_STATUS(g_status_o)

namespace thm {
namespace chunk_o {

constexpr int kThreads = 128;
constexpr int kBT = 64;  // chunk length
constexpr int kVT = 64;  // V tile per CTA

template <int K>
struct Layout {
  static constexpr int ES = 4;
  static constexpr int Q_BYTES = kBT * K * ES;       // [64 x K]  K-major
  static constexpr int V_BYTES = kBT * kVT * ES;     // [64 x VT] MN-major
  static constexpr int H_BYTES = K * kVT * 4;        // [K x VT]  MN-major fp32
  static constexpr int P_BYTES = kBT * kBT * ES;     // [64 x 64] K-major
  static constexpr int LO_Q = Q_BYTES;               // lo(q), lo(k), then lo(P)
  static constexpr int LO_V = V_BYTES;               // lo(v)
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + Q_BYTES;
  static constexpr int OFF_H = OFF_V + V_BYTES;
  static constexpr int OFF_P = OFF_H + H_BYTES;
  static constexpr int OFF_QLO = OFF_P + P_BYTES;
  static constexpr int OFF_KLO = OFF_QLO + LO_Q;
  static constexpr int OFF_VLO = OFF_KLO + LO_Q;
  static constexpr int OFF_PLO = OFF_QLO;            // lo(P) reuses lo(q)
  static constexpr int OFF_MISC = OFF_VLO + LO_V;    // g, exp(g), barriers, tmem slot
  static constexpr int MISC_BYTES = 1024;
  static constexpr int SMEM = OFF_MISC + MISC_BYTES + 1024;  // + alignment slack
  static constexpr int TX_BYTES = 2 * Q_BYTES + V_BYTES + H_BYTES;
  static constexpr uint32_t TMEM_COLS = 128;  // G [0,64) | S/L [64,128)
};

template <int K>
__global__ void __launch_bounds__(kThreads, 1)
    chunk_fwd_o_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_h,
                       const float* __restrict__ g, float* __restrict__ o, float scale, int T_len, int H, int V,
                       int NT) {
  using Ly = Layout<K>;
  constexpr int kStep = 8;  // K per tf32 MMA instruction
  constexpr uint32_t kIdS = make_idesc(2u, 64, 64, 0, 0);
  constexpr uint32_t kIdG = make_idesc(2u, 64, kVT, 0, 1);
  constexpr uint32_t kIdL = make_idesc(2u, 64, kVT, 0, 1);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(sm);
  float* sG = reinterpret_cast<float*>(sm + Ly::OFF_MISC);         // 64
  float* sEG = sG + 64;                                             // 64
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(sm + Ly::OFF_MISC + 512);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_tma + 2);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int vt = blockIdx.x;
  const int c = blockIdx.y;
  const int bh = blockIdx.z;
  const int b = bh / H;
  const int h = bh - b * H;
  const int row0 = b * T_len + c * kBT;  // first (b, t) row of the chunk
  const int v0 = vt * kVT;

  if (tid == 0) {
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_h);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, Ly::TMEM_COLS);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tG = tbase;       // columns [0, 64)
  const uint32_t tS = tbase + 64;  // columns [64, 128): S, then L

  if (tid == 0) {
    mbar_arrive_expect_tx(bar_tma, Ly::TX_BYTES);
    constexpr int kBoxK = 128 / Ly::ES;  // elements per 128-B box row
#pragma unroll
    for (int j = 0; j < K / kBoxK; ++j) {
      tma_load_3d(sm + Ly::OFF_Q + j * kBT * 128, &tm_q, bar_tma, j * kBoxK, h, row0);
      tma_load_3d(sm + Ly::OFF_K + j * kBT * 128, &tm_k, bar_tma, j * kBoxK, h, row0);
    }
#pragma unroll
    for (int j = 0; j < kVT / kBoxK; ++j)
      tma_load_3d(sm + Ly::OFF_V + j * kBT * 128, &tm_v, bar_tma, v0 + j * kBoxK, h, row0);
    const int hrow = ((b * NT + c) * H + h) * K;
#pragma unroll
    for (int j = 0; j < kVT / 32; ++j) tma_load_2d(sm + Ly::OFF_H + j * K * 128, &tm_h, bar_tma, v0 + j * 32, hrow);
  }
  if (tid < kBT) {
    const float gv = g[(long long)(row0 + tid) * H + h];
    sG[tid] = gv;
    sEG[tid] = expf(gv);
  }

  bool ok = mbar_wait(bar_tma, 0, &g_status_o);
  ok = __syncthreads_and(ok);
  if (!ok) goto cleanup_tma;

  split_tf32_tile(sm + Ly::OFF_Q, sm + Ly::OFF_QLO, Ly::Q_BYTES, tid, kThreads);
  split_tf32_tile(sm + Ly::OFF_K, sm + Ly::OFF_KLO, Ly::Q_BYTES, tid, kThreads);
  split_tf32_tile(sm + Ly::OFF_V, sm + Ly::OFF_VLO, Ly::V_BYTES, tid, kThreads);
  fence_proxy_async_smem();
  __syncthreads();

  if (tid == 0) {
    tc_fence_after();
    // S = q k^T
#pragma unroll
    for (int kk = 0; kk < K / kStep; ++kk) {
      const uint32_t kb = kk * 32;  // bytes along K
      const uint32_t off = (kb / 128) * (kBT * 128) + (kb % 128);
      const uint64_t qd = make_sdesc(sbase + Ly::OFF_Q + off, 16, 1024);
      const uint64_t kd = make_sdesc(sbase + Ly::OFF_K + off, 16, 1024);
      mma_tf32_ss(tS, qd, kd, kIdS, kk > 0);
      mma_tf32_ss(tS, qd, make_sdesc(sbase + Ly::OFF_KLO + off, 16, 1024), kIdS, 1);
      mma_tf32_ss(tS, make_sdesc(sbase + Ly::OFF_QLO + off, 16, 1024), kd, kIdS, 1);
    }
    // G = q h  (tf32; A = q, B = h MN-major)
#pragma unroll
    for (int kk = 0; kk < K / 8; ++kk) {
      const uint32_t kb = kk * 32;
      const uint32_t offa = (kb / 128) * (kBT * 128) + (kb % 128);
      mma_tf32_ss(tG, make_sdesc(sbase + Ly::OFF_Q + offa, 16, 1024),
                  make_sdesc(sbase + Ly::OFF_H + kk * 8 * 128, K * 128, 512, kSw128Base32), kIdG, kk > 0);
    }
    mma_commit(bar_mma);
  }

  ok = mbar_wait(bar_mma, 0, &g_status_o);
  ok = __syncthreads_and(ok);
  if (!ok) goto cleanup_mma0;
  tc_fence_after();

  {
    // P = tril(S * exp(g_t - g_s)) -> shared memory (A operand of P v).
    const int t = warp * 16 + lane;  // valid for lane < 16
    const uint32_t lane_addr = tS + ((uint32_t)(warp * 32) << 16);
    float srow[64];
#pragma unroll
    for (int j = 0; j < 4; ++j) tmem_ld16(lane_addr + j * 16, srow + j * 16);
    tmem_ld_wait();
    if (lane < 16) {
      const float gt = sG[t];
      uint8_t* sp = sm + Ly::OFF_P;
#pragma unroll
      for (int s0 = 0; s0 < 64; s0 += 8) {
        float pv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int s = s0 + j;
          pv[j] = (s <= t) ? srow[s] * __expf(gt - sG[s]) : 0.0f;
        }
        float hi[8], lo[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          hi[j] = tf32_round(pv[j]);
          lo[j] = pv[j] - hi[j];
        }
        uint8_t* spl = sm + Ly::OFF_PLO;
        *reinterpret_cast<float4*>(sp + sw128_offset(t, s0, kBT, 4)) = make_float4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<float4*>(sp + sw128_offset(t, s0 + 4, kBT, 4)) = make_float4(hi[4], hi[5], hi[6], hi[7]);
        *reinterpret_cast<float4*>(spl + sw128_offset(t, s0, kBT, 4)) = make_float4(lo[0], lo[1], lo[2], lo[3]);
        *reinterpret_cast<float4*>(spl + sw128_offset(t, s0 + 4, kBT, 4)) = make_float4(lo[4], lo[5], lo[6], lo[7]);
      }
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();

  if (tid == 0) {
    tc_fence_after();
    // L = P v (overwrites S's columns)
#pragma unroll
    for (int kk = 0; kk < kBT / kStep; ++kk) {
      const uint32_t kb = kk * 32;
      const uint32_t offa = (kb / 128) * (kBT * 128) + (kb % 128);
      const uint64_t ad = make_sdesc(sbase + Ly::OFF_P + offa, 16, 1024);
      const uint64_t vd = make_sdesc(sbase + Ly::OFF_V + kk * kStep * 128, kBT * 128, 512, kSw128Base32);
      const uint64_t vl = make_sdesc(sbase + Ly::OFF_VLO + kk * kStep * 128, kBT * 128, 512, kSw128Base32);
      mma_tf32_ss(tS, ad, vd, kIdL, kk > 0);
      mma_tf32_ss(tS, ad, vl, kIdL, 1);
      mma_tf32_ss(tS, make_sdesc(sbase + Ly::OFF_PLO + offa, 16, 1024), vd, kIdL, 1);
    }
    mma_commit(bar_mma);
  }
  ok = mbar_wait(bar_mma, 1, &g_status_o);
  ok = __syncthreads_and(ok);
  if (!ok) goto cleanup_mma1;
  tc_fence_after();

  {
    // o = scale * (L + exp(g_t) G)
    const int t = warp * 16 + lane;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const float eg = (lane < 16) ? sEG[t] * scale : 0.f;
    float* orow = o + ((long long)(row0 + (lane < 16 ? t : 0)) * H + h) * V + v0;
#pragma unroll
    for (int j = 0; j < kVT / 16; ++j) {
      float lv[16], gv[16];
      tmem_ld16(tS + lane_off + j * 16, lv);
      tmem_ld16(tG + lane_off + j * 16, gv);
      tmem_ld_wait();
      if (lane < 16) {
        float r[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) r[i] = fmaf(lv[i], scale, gv[i] * eg);
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          *reinterpret_cast<float4*>(orow + j * 16 + i) = make_float4(r[i], r[i + 1], r[i + 2], r[i + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, Ly::TMEM_COLS);
  return;

cleanup_mma1:
  // An MMA wait ran out of time: give the in-flight MMAs one more bounded
  // wait before releasing TMEM.
  mbar_wait(bar_mma, 1, &g_status_o);
  goto cleanup_tma;
cleanup_mma0:
  mbar_wait(bar_mma, 0, &g_status_o);
cleanup_tma:
  mbar_wait(bar_tma, 0, &g_status_o);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, Ly::TMEM_COLS);
}

template <int K>
int launch(const void* q, const void* k, const void* v, const float* g, const float* hst, void* o, float scale,
           int B, int T_len, int H, int V, cudaStream_t st) {
  using Ly = Layout<K>;
  const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const int NT = T_len / kBT;
  CUtensorMap tq, tk, tv, th;
  const uint64_t rows = (uint64_t)B * T_len;
  const uint32_t box[3] = {32u, 1u, (uint32_t)kBT};  // 128-B rows of fp32
  {
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)H, rows};
    uint64_t str[2] = {(uint64_t)K * 4, (uint64_t)H * K * 4};
    int r = encode_tiled(&tq, dt, 3, q, dims, str, box);
    if (r == THM_OK) r = encode_tiled(&tk, dt, 3, k, dims, str, box);
    if (r != THM_OK) return r;
  }
  {
    uint64_t dims[3] = {(uint64_t)V, (uint64_t)H, rows};
    uint64_t str[2] = {(uint64_t)V * 4, (uint64_t)H * V * 4};
    int r = encode_tiled(&tv, dt, 3, v, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    if (r != THM_OK) return r;
  }
  {
    uint64_t dims[2] = {(uint64_t)V, (uint64_t)B * NT * H * K};
    uint64_t str[1] = {(uint64_t)V * 4};
    uint32_t hbox[2] = {32u, (uint32_t)K};
    int r = encode_tiled(&th, dt, 2, hst, dims, str, hbox, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    if (r != THM_OK) return r;
  }
  auto kern = chunk_fwd_o_kernel<K>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Ly::SMEM) != cudaSuccess)
    return THM_ERR_CUDA;
  dim3 grid(V / kVT, NT, B * H);
  kern<<<grid, kThreads, Ly::SMEM, st>>>(tq, tk, tv, th, g, static_cast<float*>(o), scale, T_len, H, V, NT);
  return check_launch();
}


// ===========================================================================
// Persistent warp-specialized variant (bf16 q/k/v/o, bf16 h), the chain's
// kernel. One CTA per SM walks units (b, c, h) with h fastest:
//   warp 0     TMA producer: q, k, v, h tiles + gates into a 2-stage ring
//   warp 1     tcgen05 issuer (one thread), one unit ahead of the math warps:
//                S(i)    = q k^T        M=64, N=64, K=K   -> TMEM S[i%2]
//                G(i)    = q h          M=64, N=V,  K=K   -> TMEM [i%2], lane 16
//                L(i-1)  = P v          M=64, N=V,  K=64  -> TMEM [(i-1)%2], lane 0
//   warps 2-5  P(i) = tril(S * e^{g_t-g_s}) -> smem, and the epilogue
//              o = scale (L + e^{g_t} G), both with all 32 lanes through the
//              16x256b TMEM shape; o is staged in smem and written by TMA store.
// L and G are two M=64 accumulators sharing TMEM columns at lane offsets 0 and
// 16; the MN-major v and h tiles feed the tensor core straight from TMA.
// ===========================================================================
namespace ws {

constexpr int kThreads = 192;
constexpr int kMath = 128;

template <int K, int V>
struct Layout {
  static constexpr int Q_BYTES = 64 * K * 2;
  static constexpr int V_BYTES = 64 * V * 2;
  static constexpr int H_BYTES = K * V * 2;
  static constexpr int STAGE = 2 * Q_BYTES + V_BYTES + H_BYTES;
  static constexpr int OFF_Q = 0, OFF_K = Q_BYTES, OFF_V = 2 * Q_BYTES, OFF_H = 2 * Q_BYTES + V_BYTES;
  static constexpr int P_BYTES = 64 * 64 * 2;
  static constexpr int OFF_P = 2 * STAGE;
  static constexpr int OFF_O = OFF_P + 2 * P_BYTES;
  static constexpr int O_BYTES = 64 * V * 2;
  static constexpr int OFF_G = OFF_O + O_BYTES;      // gates [2][64] f32
  static constexpr int OFF_EG = OFF_G + 512;         // exp(g) [2][64] f32
  static constexpr int OFF_BAR = OFF_EG + 512;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
};

template <int K, int V>
__global__ void __launch_bounds__(kThreads, 1)
    chunk_fwd_o_ws_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_h,
                          const __grid_constant__ CUtensorMap tm_o, const float* __restrict__ g, float scale,
                          int T_len, int H, int NT, int nunits) {
  using Ly = Layout<K, V>;
  constexpr uint32_t kIdS = make_idesc(1u, 64, 64, 0, 0);
  constexpr uint32_t kIdG = make_idesc(1u, 64, V, 0, 1);
  constexpr uint32_t kIdL = make_idesc(1u, 64, V, 0, 1);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(sm);
  float* sGate = reinterpret_cast<float*>(sm + Ly::OFF_G);
  float* sEg = reinterpret_cast<float*>(sm + Ly::OFF_EG);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Ly::OFF_BAR);
  uint64_t* full = bars;        // [2] TMA stage loaded (+ gates written)
  uint64_t* empty = bars + 2;   // [2] stage consumed by the tensor core
  uint64_t* sfull = bars + 4;   // [2] S in TMEM
  uint64_t* pfull = bars + 6;   // [2] P in smem
  uint64_t* ofull = bars + 8;   // [2] L, G in TMEM
  uint64_t* tfree = bars + 10;  // [2] TMEM buffer read out
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full[i], 33);
      mbar_init(&empty[i], 1);
      mbar_init(&sfull[i], 1);
      mbar_init(&pfull[i], kMath);
      mbar_init(&ofull[i], 1);
      mbar_init(&tfree[i], kMath);
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
    int i = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++i) {
      const int st = i & 1;
      if (i >= 2) {
        ok = __all_sync(0xffffffffu, mbar_wait(&empty[st], ((i >> 1) & 1) ^ 1, &g_status_o));
        if (!ok) break;
      }
      const int hh = u % H, bc = u / H, c = bc % NT, b = bc / NT;
      const int row0 = b * T_len + c * 64;
      // the tiles first, so the gates' global-load round trip does not delay them
      if (lane == 0) {
        uint8_t* stg = sm + st * Ly::STAGE;
        mbar_arrive_expect_tx(&full[st], Ly::STAGE);
#pragma unroll
        for (int j = 0; j < K / 64; ++j) {
          tma_load_3d(stg + Ly::OFF_Q + j * 8192, &tm_q, &full[st], j * 64, hh, row0);
          tma_load_3d(stg + Ly::OFF_K + j * 8192, &tm_k, &full[st], j * 64, hh, row0);
        }
        const int hrow = ((b * NT + c) * H + hh) * K;
#pragma unroll
        for (int j = 0; j < V / 64; ++j) {
          tma_load_3d(stg + Ly::OFF_V + j * 8192, &tm_v, &full[st], j * 64, hh, row0);
          tma_load_2d(stg + Ly::OFF_H + j * K * 128, &tm_h, &full[st], j * 64, hrow);
        }
      }
      __syncwarp();
      float* gs = sGate + st * 64;
      gs[lane] = g[(long long)(row0 + lane) * H + hh];
      gs[lane + 32] = g[(long long)(row0 + lane + 32) * H + hh];
      mbar_arrive(&full[st]);
    }
  } else if (warp == 1) {
    // ---------------- tcgen05 issuer ----------------
    if (lane == 0) {
      int i = 0;
      int u = blockIdx.x;
      while (true) {
        const bool has = u < nunits;
        if (has) {
          const int st = i & 1;
          const uint32_t ph = (i >> 1) & 1;
          if (!mbar_wait(&full[st], ph, &g_status_o)) { ok = false; break; }
          if (i >= 2 && !mbar_wait(&tfree[st], ph ^ 1, &g_status_o)) { ok = false; break; }
          tc_fence_after();
          const uint32_t stg = sbase + st * Ly::STAGE;
          const uint32_t tS = tbase + 256 * st, tG = tS + 64 + (16u << 16);
#pragma unroll
          for (int kk = 0; kk < K / 16; ++kk) {
            const uint32_t off = (kk / 4) * 8192 + (kk % 4) * 32;
            mma_bf16_ss(tS, make_sdesc(stg + Ly::OFF_Q + off, 16, 1024), make_sdesc(stg + Ly::OFF_K + off, 16, 1024),
                        kIdS, kk > 0);
          }
          mma_commit(&sfull[st]);
#pragma unroll
          for (int kk = 0; kk < K / 16; ++kk) {
            const uint32_t off = (kk / 4) * 8192 + (kk % 4) * 32;
            mma_bf16_ss(tG, make_sdesc(stg + Ly::OFF_Q + off, 16, 1024),
                        make_sdesc(stg + Ly::OFF_H + kk * 2048, K * 128, 1024), kIdG, kk > 0);
          }
        }
        if (i >= 1) {
          const int j = i - 1, sj = j & 1;
          if (!mbar_wait(&pfull[sj], (j >> 1) & 1, &g_status_o)) { ok = false; break; }
          tc_fence_after();
          const uint32_t stg = sbase + sj * Ly::STAGE;
          const uint32_t tL = tbase + 256 * sj + 64;
          const uint32_t sp = sbase + Ly::OFF_P + sj * Ly::P_BYTES;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16_ss(tL, make_sdesc(sp + kk * 32, 16, 1024), make_sdesc(stg + Ly::OFF_V + kk * 2048, 8192, 1024),
                        kIdL, kk > 0);
          mma_commit(&ofull[sj]);
          mma_commit(&empty[sj]);
        }
        if (!has) break;
        ++i;
        u += gridDim.x;
      }
    }
  } else {
    // ---------------- math warps: P and epilogue ----------------
    const int mt = tid - 64;
    const int sp = warp & 3;  // TMEM subpartition this warp may access
    const uint32_t lane_base = (uint32_t)(32 * sp) << 16;
    int i = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++i) {
      const int st = i & 1;
      const uint32_t ph = (i >> 1) & 1;
      const int hh = u % H, bc = u / H, c = bc % NT, b = bc / NT;
      const int row0 = b * T_len + c * 64;
      const float* gs = sGate + st * 64;
      float* eg = sEg + st * 64;
      ok = mbar_wait(&full[st], ph, &g_status_o) && mbar_wait(&sfull[st], ph, &g_status_o);
      if (!named_bar_and(2, kMath, ok)) { ok = false; break; }
      tc_fence_after();
      {
        float sv[32];
        tmem_ld_16x256b_x8(tbase + 256 * st + lane_base, sv);
        const int r0 = 16 * sp + (lane >> 2), r1 = r0 + 8;
        const float g0 = gs[r0], g1 = gs[r1];
        uint8_t* pbuf = sm + Ly::OFF_P + st * Ly::P_BYTES;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int cc = 8 * j + 2 * (lane & 3);
          const float gc0 = gs[cc], gc1 = gs[cc + 1];
          const float p00 = (cc <= r0) ? sv[4 * j] * __expf(g0 - gc0) : 0.f;
          const float p01 = (cc + 1 <= r0) ? sv[4 * j + 1] * __expf(g0 - gc1) : 0.f;
          const float p10 = (cc <= r1) ? sv[4 * j + 2] * __expf(g1 - gc0) : 0.f;
          const float p11 = (cc + 1 <= r1) ? sv[4 * j + 3] * __expf(g1 - gc1) : 0.f;
          *reinterpret_cast<uint32_t*>(pbuf + sw128_offset(r0, cc, 64, 2)) = pack_bf16x2(p00, p01);
          *reinterpret_cast<uint32_t*>(pbuf + sw128_offset(r1, cc, 64, 2)) = pack_bf16x2(p10, p11);
        }
        if (mt < 64) eg[mt] = __expf(gs[mt]) * scale;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&pfull[st]);

      ok = mbar_wait(&ofull[st], ph, &g_status_o);
      if (!named_bar_and(2, kMath, ok)) { ok = false; break; }
      tc_fence_after();
      if (mt == 0) bulk_wait_group_read0();  // previous o tile has left smem
      named_bar_sync(1, kMath);
      {
        // o = scale L + e^{g_t} scale G for rows r0, r0 + 8, packed bf16 pairs
        const int r0 = 16 * sp + (lane >> 2), r1 = r0 + 8;
        const float e0 = eg[r0], e1 = eg[r1];
        const uint32_t swz = (uint32_t)((lane >> 2) & 7);
        const uint32_t tL = tbase + 256 * st + 64 + lane_base;
#pragma unroll
        for (int half = 0; half < V / 64; ++half) {
          float lv[32], gv[32];
          tmem_ld_16x256b_x8(tL + 64 * half, lv);
          tmem_ld_16x256b_x8(tL + (16u << 16) + 64 * half, gv);
          uint8_t* box = sm + Ly::OFF_O + half * 8192;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t off = (((uint32_t)j ^ swz) << 4) + (uint32_t)(lane & 3) * 4;
            *reinterpret_cast<uint32_t*>(box + r0 * 128 + off) =
                pack_bf16x2(fmaf(lv[4 * j], scale, gv[4 * j] * e0), fmaf(lv[4 * j + 1], scale, gv[4 * j + 1] * e0));
            *reinterpret_cast<uint32_t*>(box + r1 * 128 + off) =
                pack_bf16x2(fmaf(lv[4 * j + 2], scale, gv[4 * j + 2] * e1), fmaf(lv[4 * j + 3], scale, gv[4 * j + 3] * e1));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tfree[st]);
      fence_proxy_async_smem();
      named_bar_sync(1, kMath);
      if (mt == 0) {
#pragma unroll
        for (int j = 0; j < V / 64; ++j) tma_store_3d(&tm_o, sm + Ly::OFF_O + j * 8192, j * 64, hh, row0);
        bulk_commit_group();
      }
    }
    if (mt == 0) bulk_wait_group0();
  }

  if (!ok) record_status(&g_status_o, THM_ERR_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 512);
}

template <int K, int V>
int launch(const void* q, const void* k, const void* v, const float* g, const void* hst, void* o, float scale,
           int B, int T_len, int H, cudaStream_t st) {
  using Ly = Layout<K, V>;
  const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int NT = T_len / 64;
  const uint64_t rows = (uint64_t)B * T_len;
  const uint32_t box[3] = {64u, 1u, 64u};
  CUtensorMap tq, tk, tv, th, to;
  {
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)H, rows};
    uint64_t str[2] = {(uint64_t)K * 2, (uint64_t)H * K * 2};
    int r = encode_tiled(&tq, dt, 3, q, dims, str, box);
    if (r == THM_OK) r = encode_tiled(&tk, dt, 3, k, dims, str, box);
    if (r != THM_OK) return r;
  }
  {
    uint64_t dims[3] = {(uint64_t)V, (uint64_t)H, rows};
    uint64_t str[2] = {(uint64_t)V * 2, (uint64_t)H * V * 2};
    int r = encode_tiled(&tv, dt, 3, v, dims, str, box);
    if (r == THM_OK) r = encode_tiled(&to, dt, 3, o, dims, str, box);
    if (r != THM_OK) return r;
  }
  {
    uint64_t dims[2] = {(uint64_t)V, (uint64_t)B * NT * H * K};
    uint64_t str[1] = {(uint64_t)V * 2};
    uint32_t hbox[2] = {64u, (uint32_t)K};
    int r = encode_tiled(&th, dt, 2, hst, dims, str, hbox);
    if (r != THM_OK) return r;
  }
  auto kern = chunk_fwd_o_ws_kernel<K, V>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Ly::SMEM) != cudaSuccess)
    return THM_ERR_CUDA;
  const int nunits = B * NT * H;
  const int grid = nunits < sm_count() ? nunits : sm_count();
  kern<<<grid, kThreads, Ly::SMEM, st>>>(tq, tk, tv, th, to, g, scale, T_len, H, NT, nunits);
  return check_launch();
}

}  // namespace ws

// ===========================================================================
// Persistent warp-specialized variant for bf16 q/k/v/o with fp32 states h
// (the reference's h is fp32). Units are (b, c, h, 64-column
// V tile) with the V tile fastest, so the tiles of one (b, c, h) run on
// neighbouring CTAs at the same time and share the q, k lines through L2.
//
// The fp32 h tile is split on the fly into two bf16 tiles, hi = bf16(h) and
// lo = bf16(h - hi), and G = q hi + q lo runs in kind::f16. q is exact in bf16,
// so G carries about 16 significant bits of h (|h - hi - lo| <= 2^-16 |h|),
// more than the 10 of a tf32 product, at the tensor cost of one tf32 product.
//   warp 0     TMA producer: q, k, v tile, fp32 h tile + gates, 2-stage ring
//   warp 1     tcgen05 issuer (one thread), per unit i:
//                L(i-1) = P v       once P(i-1) is in smem
//                S(i)   = q k^T     M=64, N=64, K=K   -> TMEM [i%2] cols 0..63
//                G(i)   = q hi + q lo once hi/lo(i) is in smem -> [i%2] lane 16
//   warps 2-5  P(i) = tril(S e^{g_t-g_s}) and the epilogue o = scale (L + e^{g_t} G)
//   warps 6-9  hi/lo(i) from the fp32 tile (single buffer, freed by G(i-1))
// ===========================================================================
namespace ws32 {

constexpr int kThreads = 320;
constexpr int kMath = 128;
constexpr int kConv = 128;
constexpr int kVT = 64;

template <int K>
struct Layout {
  static constexpr int Q_BYTES = 64 * K * 2;          // [64 x K] bf16, K-major SW128
  static constexpr int V_BYTES = 64 * kVT * 2;        // [64 x 64] bf16, MN-major SW128
  static constexpr int H32_BYTES = K * kVT * 4;       // [K x 64] fp32, row-major (no swizzle)
  static constexpr int OFF_Q = 0, OFF_K = Q_BYTES, OFF_V = 2 * Q_BYTES, OFF_H32 = 2 * Q_BYTES + V_BYTES;
  static constexpr int STAGE = OFF_H32 + H32_BYTES;
  static constexpr int HL_BYTES = K * kVT * 2;        // [K x 64] bf16, MN-major SW128
  static constexpr int OFF_HI = 2 * STAGE, OFF_LO = OFF_HI + HL_BYTES;
  static constexpr int P_BYTES = 64 * 64 * 2;
  static constexpr int OFF_P = OFF_LO + HL_BYTES;
  static constexpr int O_BYTES = 64 * kVT * 2;
  static constexpr int OFF_O = OFF_P + 2 * P_BYTES;
  static constexpr int OFF_G = OFF_O + O_BYTES;       // gates [2][64] f32
  static constexpr int OFF_EG = OFF_G + 512;          // scale e^g [2][64] f32
  static constexpr int OFF_BAR = OFF_EG + 512;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static_assert(STAGE % 1024 == 0 && HL_BYTES % 1024 == 0, "1024-B aligned tiles");
};

template <int K>
__global__ void __launch_bounds__(kThreads, 1)
    chunk_fwd_o_ws32_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                            const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_h,
                            const __grid_constant__ CUtensorMap tm_o, const float* __restrict__ g, float scale,
                            int T_len, int H, int NT, int NVT, int nunits) {
  using Ly = Layout<K>;
  constexpr uint32_t kIdS = make_idesc(1u, 64, 64, 0, 0);
  constexpr uint32_t kIdG = make_idesc(1u, 64, kVT, 0, 1);
  constexpr uint32_t kIdL = make_idesc(1u, 64, kVT, 0, 1);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(sm);
  float* sGate = reinterpret_cast<float*>(sm + Ly::OFF_G);
  float* sEg = reinterpret_cast<float*>(sm + Ly::OFF_EG);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Ly::OFF_BAR);
  uint64_t* full = bars;        // [2] TMA stage loaded (+ gates written)
  uint64_t* empty = bars + 2;   // [2] stage consumed (tensor core and converters)
  uint64_t* sfull = bars + 4;   // [2] S in TMEM
  uint64_t* pfull = bars + 6;   // [2] P in smem
  uint64_t* ofull = bars + 8;   // [2] L, G in TMEM
  uint64_t* tfree = bars + 10;  // [2] TMEM buffer read out
  uint64_t* hready = bars + 12; // hi/lo tiles written
  uint64_t* gdone = bars + 13;  // G read the hi/lo tiles
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full[i], 33);
      mbar_init(&empty[i], 1);
      mbar_init(&sfull[i], 1);
      mbar_init(&pfull[i], kMath);
      mbar_init(&ofull[i], 1);
      mbar_init(&tfree[i], kMath);
    }
    mbar_init(hready, kConv);
    mbar_init(gdone, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    int i = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++i) {
      const int st = i & 1;
      if (i >= 2) {
        ok = __all_sync(0xffffffffu, mbar_wait(&empty[st], ((i >> 1) & 1) ^ 1, &g_status_o));
        if (!ok) break;
      }
      const int vt = u % NVT, r = u / NVT, hh = r % H, bc = r / H, c = bc % NT, b = bc / NT;
      const int row0 = b * T_len + c * 64;
      // the tiles first, so the gates' global-load round trip does not delay them
      if (lane == 0) {
        uint8_t* stg = sm + st * Ly::STAGE;
        mbar_arrive_expect_tx(&full[st], Ly::STAGE);
#pragma unroll
        for (int j = 0; j < K / 64; ++j) {
          tma_load_3d(stg + Ly::OFF_Q + j * 8192, &tm_q, &full[st], j * 64, hh, row0);
          tma_load_3d(stg + Ly::OFF_K + j * 8192, &tm_k, &full[st], j * 64, hh, row0);
        }
        tma_load_3d(stg + Ly::OFF_V, &tm_v, &full[st], vt * kVT, hh, row0);
        tma_load_2d(stg + Ly::OFF_H32, &tm_h, &full[st], vt * kVT, ((b * NT + c) * H + hh) * K);
      }
      __syncwarp();
      float* gs = sGate + st * 64;
      gs[lane] = g[(long long)(row0 + lane) * H + hh];
      gs[lane + 32] = g[(long long)(row0 + lane + 32) * H + hh];
      mbar_arrive(&full[st]);
    }
  } else if (warp == 1) {
    // ---------------- tcgen05 issuer ----------------
    if (lane == 0) {
      int i = 0;
      int u = blockIdx.x;
      while (true) {
        const bool has = u < nunits;
        if (i >= 1) {
          // L(i-1) = P v: frees the stage of unit i-1 when done.
          const int j = i - 1, sj = j & 1;
          if (!mbar_wait(&pfull[sj], (j >> 1) & 1, &g_status_o)) { ok = false; break; }
          tc_fence_after();
          const uint32_t stg = sbase + sj * Ly::STAGE;
          const uint32_t tL = tbase + 128 * sj + 64;
          const uint32_t sp = sbase + Ly::OFF_P + sj * Ly::P_BYTES;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16_ss(tL, make_sdesc(sp + kk * 32, 16, 1024), make_sdesc(stg + Ly::OFF_V + kk * 2048, 8192, 1024),
                        kIdL, kk > 0);
          mma_commit(&ofull[sj]);
          mma_commit(&empty[sj]);
        }
        if (!has) break;
        const int st = i & 1;
        const uint32_t ph = (i >> 1) & 1;
        if (!mbar_wait(&full[st], ph, &g_status_o)) { ok = false; break; }
        if (i >= 2 && !mbar_wait(&tfree[st], ph ^ 1, &g_status_o)) { ok = false; break; }
        tc_fence_after();
        const uint32_t stg = sbase + st * Ly::STAGE;
        const uint32_t tS = tbase + 128 * st, tG = tS + 64 + (16u << 16);
#pragma unroll
        for (int kk = 0; kk < K / 16; ++kk) {
          const uint32_t off = (kk / 4) * 8192 + (kk % 4) * 32;
          mma_bf16_ss(tS, make_sdesc(stg + Ly::OFF_Q + off, 16, 1024), make_sdesc(stg + Ly::OFF_K + off, 16, 1024),
                      kIdS, kk > 0);
        }
        mma_commit(&sfull[st]);
        if (!mbar_wait(hready, i & 1, &g_status_o)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < K / 16; ++kk) {
          const uint64_t qd = make_sdesc(stg + Ly::OFF_Q + (kk / 4) * 8192 + (kk % 4) * 32, 16, 1024);
          mma_bf16_ss(tG, qd, make_sdesc(sbase + Ly::OFF_HI + kk * 2048, Ly::HL_BYTES, 1024), kIdG, kk > 0);
          mma_bf16_ss(tG, qd, make_sdesc(sbase + Ly::OFF_LO + kk * 2048, Ly::HL_BYTES, 1024), kIdG, 1);
        }
        mma_commit(gdone);
        ++i;
        u += gridDim.x;
      }
    }
  } else if (warp < 6) {
    // ---------------- math warps: P and epilogue ----------------
    const int mt = tid - 64;
    const int sp = warp & 3;  // TMEM subpartition this warp may access
    const uint32_t lane_base = (uint32_t)(32 * sp) << 16;
    int i = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++i) {
      const int st = i & 1;
      const uint32_t ph = (i >> 1) & 1;
      const int vt = u % NVT, r = u / NVT, hh = r % H, bc = r / H, c = bc % NT, b = bc / NT;
      const int row0 = b * T_len + c * 64;
      const float* gs = sGate + st * 64;
      float* eg = sEg + st * 64;
      ok = mbar_wait(&full[st], ph, &g_status_o) && mbar_wait(&sfull[st], ph, &g_status_o);
      if (!named_bar_and(2, kMath, ok)) { ok = false; break; }
      tc_fence_after();
      {
        float sv[32];
        tmem_ld_16x256b_x8(tbase + 128 * st + lane_base, sv);
        const int r0 = 16 * sp + (lane >> 2), r1 = r0 + 8;
        const float g0 = gs[r0], g1 = gs[r1];
        uint8_t* pbuf = sm + Ly::OFF_P + st * Ly::P_BYTES;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int cc = 8 * j + 2 * (lane & 3);
          const float gc0 = gs[cc], gc1 = gs[cc + 1];
          const float p00 = (cc <= r0) ? sv[4 * j] * __expf(g0 - gc0) : 0.f;
          const float p01 = (cc + 1 <= r0) ? sv[4 * j + 1] * __expf(g0 - gc1) : 0.f;
          const float p10 = (cc <= r1) ? sv[4 * j + 2] * __expf(g1 - gc0) : 0.f;
          const float p11 = (cc + 1 <= r1) ? sv[4 * j + 3] * __expf(g1 - gc1) : 0.f;
          *reinterpret_cast<uint32_t*>(pbuf + sw128_offset(r0, cc, 64, 2)) = pack_bf16x2(p00, p01);
          *reinterpret_cast<uint32_t*>(pbuf + sw128_offset(r1, cc, 64, 2)) = pack_bf16x2(p10, p11);
        }
        if (mt < 64) eg[mt] = __expf(gs[mt]) * scale;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&pfull[st]);

      ok = mbar_wait(&ofull[st], ph, &g_status_o);
      if (!named_bar_and(2, kMath, ok)) { ok = false; break; }
      tc_fence_after();
      if (mt == 0) bulk_wait_group_read0();  // previous o tile has left smem
      named_bar_sync(1, kMath);
      {
        // o = scale L + e^{g_t} scale G for rows r0, r0 + 8, packed bf16 pairs
        const int r0 = 16 * sp + (lane >> 2), r1 = r0 + 8;
        const float e0 = eg[r0], e1 = eg[r1];
        const uint32_t swz = (uint32_t)((lane >> 2) & 7);
        const uint32_t tL = tbase + 128 * st + 64 + lane_base;
        float lv[32], gv[32];
        tmem_ld_16x256b_x8(tL, lv);
        tmem_ld_16x256b_x8(tL + (16u << 16), gv);
        uint8_t* box = sm + Ly::OFF_O;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t off = (((uint32_t)j ^ swz) << 4) + (uint32_t)(lane & 3) * 4;
          *reinterpret_cast<uint32_t*>(box + r0 * 128 + off) =
              pack_bf16x2(fmaf(lv[4 * j], scale, gv[4 * j] * e0), fmaf(lv[4 * j + 1], scale, gv[4 * j + 1] * e0));
          *reinterpret_cast<uint32_t*>(box + r1 * 128 + off) =
              pack_bf16x2(fmaf(lv[4 * j + 2], scale, gv[4 * j + 2] * e1), fmaf(lv[4 * j + 3], scale, gv[4 * j + 3] * e1));
        }
      }
      tc_fence_before();
      mbar_arrive(&tfree[st]);
      fence_proxy_async_smem();
      named_bar_sync(1, kMath);
      if (mt == 0) {
        tma_store_3d(&tm_o, sm + Ly::OFF_O, vt * kVT, hh, row0);
        bulk_commit_group();
      }
    }
    if (mt == 0) bulk_wait_group0();
  } else {
    // ---------------- converters: fp32 h tile -> bf16 hi, lo ----------------
    const int ct = tid - 192;
    uint8_t* hi = sm + Ly::OFF_HI;
    uint8_t* lo = sm + Ly::OFF_LO;
    int i = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++i) {
      const int st = i & 1;
      ok = mbar_wait(&full[st], (i >> 1) & 1, &g_status_o) && (i == 0 || mbar_wait(gdone, (i - 1) & 1, &g_status_o));
      if (!named_bar_and(3, kConv, ok)) { ok = false; break; }
      const float* h32 = reinterpret_cast<const float*>(sm + st * Ly::STAGE + Ly::OFF_H32);
#pragma unroll 4
      for (int it = 0; it < K * kVT / 4 / kConv; ++it) {
        const int idx = it * kConv + ct;           // float4 index: 16 per 64-column row
        const int rr = idx >> 4, c4 = (idx & 15) * 4;
        const float4 x = *reinterpret_cast<const float4*>(h32 + rr * kVT + c4);
        const __nv_bfloat162 h01 = __floats2bfloat162_rn(x.x, x.y), h23 = __floats2bfloat162_rn(x.z, x.w);
        const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
        const __nv_bfloat162 l01 = __floats2bfloat162_rn(x.x - f01.x, x.y - f01.y);
        const __nv_bfloat162 l23 = __floats2bfloat162_rn(x.z - f23.x, x.w - f23.y);
        const uint32_t off = sw128_offset(rr, c4, K, 2);
        *reinterpret_cast<uint2*>(hi + off) =
            make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
        *reinterpret_cast<uint2*>(lo + off) =
            make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
      }
      fence_proxy_async_smem();
      mbar_arrive(hready);
    }
  }

  if (!ok) record_status(&g_status_o, THM_ERR_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 256);
}

template <int K>
int launch(const void* q, const void* k, const void* v, const float* g, const float* hst, void* o, float scale,
           int B, int T_len, int H, int V, cudaStream_t st) {
  using Ly = Layout<K>;
  const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int NT = T_len / 64;
  const uint64_t rows = (uint64_t)B * T_len;
  const uint32_t box[3] = {64u, 1u, 64u};
  CUtensorMap tq, tk, tv, th, to;
  {
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)H, rows};
    uint64_t str[2] = {(uint64_t)K * 2, (uint64_t)H * K * 2};
    int r = encode_tiled(&tq, dt, 3, q, dims, str, box);
    if (r == THM_OK) r = encode_tiled(&tk, dt, 3, k, dims, str, box);
    if (r != THM_OK) return r;
  }
  {
    uint64_t dims[3] = {(uint64_t)V, (uint64_t)H, rows};
    uint64_t str[2] = {(uint64_t)V * 2, (uint64_t)H * V * 2};
    int r = encode_tiled(&tv, dt, 3, v, dims, str, box);
    if (r == THM_OK) r = encode_tiled(&to, dt, 3, o, dims, str, box);
    if (r != THM_OK) return r;
  }
  {
    uint64_t dims[2] = {(uint64_t)V, (uint64_t)B * NT * H * K};
    uint64_t str[1] = {(uint64_t)V * 4};
    uint32_t hbox[2] = {(uint32_t)kVT, (uint32_t)K};
    int r = encode_tiled(&th, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, hst, dims, str, hbox, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (r != THM_OK) return r;
  }
  auto kern = chunk_fwd_o_ws32_kernel<K>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Ly::SMEM) != cudaSuccess)
    return THM_ERR_CUDA;
  const int NVT = V / kVT;
  const long long nu = (long long)B * NT * H * NVT;
  if (nu > 0x7fffffffLL) return THM_ERR_UNSUPPORTED;
  const int nunits = (int)nu;
  const int grid = nunits < sm_count() ? nunits : sm_count();
  kern<<<grid, kThreads, Ly::SMEM, st>>>(tq, tk, tv, th, to, g, scale, T_len, H, NT, NVT, nunits);
  return check_launch();
}

}  // namespace ws32
}  // namespace chunk_o
}  // namespace thm

THM_STATUS_READER(thm_internal_status_o, g_status_o)

extern "C" int thm_chunk_fwd_o_fwd(const void* q, const void* k, const void* v, const float* g, const void* h,
                                   void* o, float scale, int B, int T, int H, int K, int V, int dtype, int h_dtype,
                                   thm_stream_t stream) {
  using namespace thm;
  if (B < 0 || T < 0 || H < 0 || K <= 0 || V <= 0) return THM_ERR_INVALID;
  if (T % 64 != 0) return THM_ERR_INVALID;
  if (dtype != THM_F32 && dtype != THM_BF16) return THM_ERR_INVALID;
  if (h_dtype != THM_F32 && h_dtype != THM_BF16) return THM_ERR_INVALID;
  if ((long long)B * T * H == 0) return THM_OK;
  if (!q || !k || !v || !g || !h || !o) return THM_ERR_INVALID;
  if (!(K == 64 || K == 128) || V % 64 != 0 || V > 512) return THM_ERR_UNSUPPORTED;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(h) || !aligned16(o)) return THM_ERR_ALIGNMENT;
  if ((long long)B * H > 65535 || T / 64 > 65535) return THM_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (h_dtype == THM_BF16) {
    // bf16 state: the persistent warp-specialized kernel (bf16 activations).
    if (dtype != THM_BF16 || !(V == 64 || V == 128)) return THM_ERR_UNSUPPORTED;
    if (K == 64)
      return V == 64 ? chunk_o::ws::launch<64, 64>(q, k, v, g, h, o, scale, B, T, H, st)
                     : chunk_o::ws::launch<64, 128>(q, k, v, g, h, o, scale, B, T, H, st);
    return V == 64 ? chunk_o::ws::launch<128, 64>(q, k, v, g, h, o, scale, B, T, H, st)
                   : chunk_o::ws::launch<128, 128>(q, k, v, g, h, o, scale, B, T, H, st);
  }
  const float* hf = static_cast<const float*>(h);
  if (dtype == THM_BF16) {
    // fp32 state, bf16 activations: persistent kernel with the hi/lo split of h.
    return K == 64 ? chunk_o::ws32::launch<64>(q, k, v, g, hf, o, scale, B, T, H, V, st)
                   : chunk_o::ws32::launch<128>(q, k, v, g, hf, o, scale, B, T, H, V, st);
  }
  return K == 64 ? chunk_o::launch<64>(q, k, v, g, hf, o, scale, B, T, H, V, st)
                 : chunk_o::launch<128>(q, k, v, g, hf, o, scale, B, T, H, V, st);
}
