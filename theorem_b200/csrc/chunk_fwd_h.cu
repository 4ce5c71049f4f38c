// chunk_fwd_h.cu -- inter-chunk state recurrence on tcgen05 tensor cores.
//
// Replaces kernels/chunk_fwd_h/kernel.py:61-138 (chunk_fwd_h_kernel) and its
// launcher :141-191. One CTA (128 threads) per (b, h, 64-wide V tile) walks
// the chunks of its sequence in order; the fp32 state tile S [K x 64] lives in
// registers (thread <-> row of S) for the whole sequence, so it never leaves
// the SM except as the h output.
//
// mode 0 (reference, kernels/chunk_fwd_h/reference.py:75-95):
//   U_c = k_c^T (v_c * exp(g_last - g_c))      tensor core (M=K, N=64, K=64)
//   S   = exp(g_last) S + U_c ;  h[c] = S      registers
// mode 1 (gated delta rule, state entering the chunk stored as h[c]):
//   h[c] = S;  S -> smem (bf16 / tf32) as an MMA operand
//   X     = w_c S                               tensor core (M=64, N=64, K=K)
//   v_new = u_c - X  (-> HBM if requested)      registers
//   U_c   = k_c^T (v_new * exp(g_last - g_c))   tensor core (M=K, N=64, K=64)
//   S     = exp(g_last) S + U_c                 registers
//
// k, v/u (and w) tiles of chunk c+2 stream in by TMA (double-buffered, 128-B
// swizzle; 32-B atoms for MN-major tf32 operands) while chunk c is processed;
// the h and v_new tiles leave through shared memory by TMA store (a row per
// thread written straight to HBM would touch 32 rows per store instruction).
#include <cuda_bf16.h>

#include <type_traits>

#include "host_util.h"
#include "sm100.cuh"

THM_DEFINE_STATUS(g_status_h)

namespace thm {
namespace chunk_h {

constexpr int kThreads = 128;
constexpr int kBT = 64;
constexpr int kVT = 64;
constexpr int kStoreVn = 1;  // flags: v_new is written
constexpr int kStoreH = 2;   // flags: h is written (always in mode 0)

template <typename T, int K, int MODE, bool HB>
struct Layout {
  static constexpr int ES = sizeof(T);
  static constexpr bool BF16 = ES == 2;
  static constexpr int HES = HB ? 2 : 4;                      // stored h element size
  static constexpr int K_BYTES = kBT * K * ES;               // k_c: MN-major A (k^T)
  static constexpr int V_BYTES = kBT * kVT * ES;             // v_c / u_c: MN-major B
  static constexpr int W_BYTES = MODE == 1 ? kBT * K * ES : 0;  // w_c: K-major A
  static constexpr int STAGE = K_BYTES + V_BYTES + W_BYTES;
  static constexpr int S_BYTES = MODE == 1 ? K * kVT * ES : 0;  // state as MN-major B
  // The stored h tile leaves by TMA store. In delta mode with h in the
  // activation dtype it is the MMA copy of the state itself; otherwise a
  // separate [K x 64] staging tile (128-B swizzle, 16-B chunks).
  static constexpr bool H_FROM_S = MODE == 1 && (HES == ES);
  static constexpr int HST_BYTES = H_FROM_S ? 0 : K * kVT * HES;
  static constexpr int VN_BYTES = MODE == 1 ? kBT * kVT * ES : 0;  // v_new staging
  static constexpr int OFF_STAGE0 = 0;
  static constexpr int OFF_S = 2 * STAGE;
  static constexpr int OFF_HST = OFF_S + S_BYTES;
  static constexpr int OFF_VN = OFF_HST + HST_BYTES;
  static constexpr int OFF_MISC = OFF_VN + VN_BYTES;
  // misc: sG [2][64] | decay factors [64] | barriers, TMEM slot
  static constexpr int SMEM = OFF_MISC + 2048 + 1024;
  static constexpr uint32_t TMEM_COLS = 128;  // U [0,64) | X [64,128)
};

// Write one 64-wide state row (fp32 registers) into a [rows x 64] tile of
// element type E, 128-B swizzle: 16-B chunks (layout 2) or 32-B atoms (layout 1).
template <typename E, bool ATOM32>
__device__ __forceinline__ void write_state_row(uint8_t* tile, int row, int rows, const float* S) {
  if constexpr (sizeof(E) == 2) {
#pragma unroll
    for (int j = 0; j < kVT; j += 8) {
      uint4 p;
      p.x = pack_bf16x2(S[j], S[j + 1]);
      p.y = pack_bf16x2(S[j + 2], S[j + 3]);
      p.z = pack_bf16x2(S[j + 4], S[j + 5]);
      p.w = pack_bf16x2(S[j + 6], S[j + 7]);
      *reinterpret_cast<uint4*>(tile + sw128_offset(row, j, rows, 2)) = p;
    }
  } else {
#pragma unroll
    for (int j = 0; j < kVT; j += 4) {
      const uint32_t off = ATOM32 ? sw128b32_offset(row, j, rows, 4) : sw128_offset(row, j, rows, 4);
      *reinterpret_cast<float4*>(tile + off) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
    }
  }
}

template <typename T, int K, int MODE, bool HB>
__global__ void __launch_bounds__(kThreads, 1)
    chunk_fwd_h_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                       const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_hst,
                       const __grid_constant__ CUtensorMap tm_vn, const float* __restrict__ g,
                       const float* __restrict__ h0, float* __restrict__ final_state, int flags, int T_len,
                       int H, int V) {
  using Ly = Layout<T, K, MODE, HB>;
  using HT = typename std::conditional<HB, __nv_bfloat16, float>::type;
  constexpr bool kBf16 = Ly::BF16;
  constexpr uint32_t kFmt = kBf16 ? 1u : 2u;
  constexpr int kStep = kBf16 ? 16 : 8;
  constexpr uint32_t kMNLayout = kBf16 ? kSw128 : kSw128Base32;  // MN-major operands
  constexpr uint32_t kMNSbo = kBf16 ? 1024u : 512u;
  constexpr uint32_t kIdU = make_idesc(kFmt, K, kVT, 1, 1);
  constexpr uint32_t kIdX = make_idesc(kFmt, 64, kVT, 0, 1);
  constexpr int kBox = 128 / Ly::ES;
  constexpr int kHBox = 128 / Ly::HES;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(sm);
  float* sG = reinterpret_cast<float*>(sm + Ly::OFF_MISC);         // [2][64]
  float* sFac = reinterpret_cast<float*>(sm + Ly::OFF_MISC + 512);  // [64]
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(sm + Ly::OFF_MISC + 1024);  // [2]
  uint64_t* bar_mma = bar_tma + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_tma + 4);
  uint8_t* hst = sm + (Ly::H_FROM_S ? Ly::OFF_S : Ly::OFF_HST);  // tile the h store reads

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int vt = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / H, hh = bh - (bh / H) * H;
  const int v0 = vt * kVT;
  const int NT = T_len / kBT;
  // Row of S this thread owns (M = K layout in TMEM).
  const bool srow_ok = (K == 128) || lane < 16;
  const int kk = (K == 128) ? tid : warp * 16 + lane;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;

  auto issue_tma = [&](int c, int st) {
    uint8_t* base = sm + Ly::OFF_STAGE0 + st * Ly::STAGE;
    const int row0 = b * T_len + c * kBT;
    mbar_arrive_expect_tx(&bar_tma[st], Ly::STAGE);
#pragma unroll
    for (int j = 0; j < K / kBox; ++j) {
      tma_load_3d(base + j * kBT * 128, &tm_k, &bar_tma[st], j * kBox, hh, row0);
      if (MODE == 1) tma_load_3d(base + Ly::K_BYTES + Ly::V_BYTES + j * kBT * 128, &tm_w, &bar_tma[st], j * kBox, hh, row0);
    }
#pragma unroll
    for (int j = 0; j < kVT / kBox; ++j)
      tma_load_3d(base + Ly::K_BYTES + j * kBT * 128, &tm_v, &bar_tma[st], v0 + j * kBox, hh, row0);
  };
  // TMA store of the h tile of chunk c (bulk group; waited before reuse).
  auto store_h = [&](int c) {
    const int hrow = ((b * NT + c) * H + hh) * K;
#pragma unroll
    for (int j = 0; j < kVT / kHBox; ++j) tma_store_2d(&tm_hst, hst + j * K * 128, v0 + j * kHBox, hrow);
  };

  if (tid == 0) {
    mbar_init(&bar_tma[0], 1);
    mbar_init(&bar_tma[1], 1);
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
  const uint32_t tU = tbase, tX = tbase + 64;

  if (tid == 0) {
    issue_tma(0, 0);
    if (NT > 1) issue_tma(1, 1);
  }
  if (tid < kBT) {
    sG[tid] = g[(long long)(b * T_len + tid) * H + hh];
    if (NT > 1) sG[64 + tid] = g[(long long)(b * T_len + kBT + tid) * H + hh];
  }

  float S[kVT];
#pragma unroll
  for (int j = 0; j < kVT; ++j) S[j] = 0.f;
  if (MODE == 1 && h0 != nullptr && srow_ok) {
    const float* src = h0 + (((long long)b * H + hh) * K + kk) * V + v0;
#pragma unroll
    for (int j = 0; j < kVT; j += 4) {
      const float4 x = *reinterpret_cast<const float4*>(src + j);
      S[j] = x.x; S[j + 1] = x.y; S[j + 2] = x.z; S[j + 3] = x.w;
    }
  }
  __syncthreads();

  uint32_t mphase = 0;
  int pending = -1;           // parity of an MMA commit not yet waited for
  int last_issued = (NT > 1) ? 1 : 0;  // highest chunk whose TMA was issued
  int consumed = -1;          // highest chunk whose TMA wait succeeded
  bool ok = true;
  for (int c = 0; c < NT; ++c) {
    const int st = c & 1;
    uint8_t* stage = sm + Ly::OFF_STAGE0 + st * Ly::STAGE;
    const uint32_t sk = sbase + Ly::OFF_STAGE0 + st * Ly::STAGE;  // k tile
    const uint32_t sv = sk + Ly::K_BYTES;                           // v / u tile
    const uint32_t sw = sv + Ly::V_BYTES;                           // w tile
    const float* gc = sG + st * 64;
    const int row0 = b * T_len + c * kBT;

    if constexpr (MODE == 1) {
      // The previous chunk's h / v_new tiles have left shared memory.
      if (tid == 0) bulk_wait_group_read0();
      __syncthreads();
      // h[c] = state entering chunk c. S -> smem as the B operand of X = w S
      // (and, when h is stored in the activation dtype, as the h tile).
      if (srow_ok) {
        write_state_row<T, !kBf16>(sm + Ly::OFF_S, kk, K, S);
        if constexpr (!Ly::H_FROM_S) write_state_row<HT, false>(sm + Ly::OFF_HST, kk, K, S);
      }
      fence_proxy_async_smem();
      tc_fence_before();
    }
    cp_async_wait<1>();  // this chunk's gates (committed two steps ago) have landed
    ok = mbar_wait(&bar_tma[st], (c >> 1) & 1, &g_status_h);
    ok = __syncthreads_and(ok);
    if (!ok) break;
    consumed = c;
    const float gl = gc[kBT - 1];

    if constexpr (MODE == 1) {
      if (tid == 0) {
        if (flags & kStoreH) store_h(c);
        tc_fence_after();
#pragma unroll
        for (int q = 0; q < K / kStep; ++q) {
          const uint32_t kb = q * 32;
          const uint64_t ad = make_sdesc(sw + (kb / 128) * (kBT * 128) + (kb % 128), 16, 1024);
          const uint64_t bd = make_sdesc(sbase + Ly::OFF_S + q * kStep * 128, K * 128, kMNSbo, kMNLayout);
          mma_kind<kBf16>(tX, ad, bd, kIdX, q > 0);
        }
        mma_commit(bar_mma);
      }
      pending = (int)mphase;
      ok = mbar_wait(bar_mma, mphase, &g_status_h);
      mphase ^= 1;
      ok = __syncthreads_and(ok);
      if (!ok) break;
      pending = -1;
      tc_fence_after();
      // v_new = u - X -> staging tile; u tile <- v_new * exp(g_last - g_t)
      {
        float xr[kVT];
        tmem_ld64(tX + lane_off, xr);  // one 64-column load, one wait
        if (lane < 16) {
          const int t = warp * 16 + lane;
          const float dec = __expf(gl - gc[t]);
          uint8_t* vn = sm + Ly::OFF_VN;
#pragma unroll
          for (int j = 0; j < kVT; j += 8) {
            float un[8];
            if constexpr (kBf16) {
              uint4* p = reinterpret_cast<uint4*>(stage + Ly::K_BYTES + sw128_offset(t, j, kBT, 2));
              uint4 r = *p;
              const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&r);
              uint32_t o4[4], s4[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                // u - x as fma(x, -1, u) and the decayed copy, packed fp32x2 (same roundings)
                const float2 f = __bfloat1622float2(h2[q]);
                const float2 d2 = __ffma2_rn(make_float2(xr[j + 2 * q], xr[j + 2 * q + 1]), make_float2(-1.f, -1.f), f);
                const float2 e2 = __fmul2_rn(d2, make_float2(dec, dec));
                un[2 * q] = d2.x;
                un[2 * q + 1] = d2.y;
                o4[q] = pack_bf16x2(d2.x, d2.y);
                s4[q] = pack_bf16x2(e2.x, e2.y);
              }
              *reinterpret_cast<uint4*>(vn + sw128_offset(t, j, kBT, 2)) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
              *p = make_uint4(s4[0], s4[1], s4[2], s4[3]);
            } else {
#pragma unroll
              for (int q = 0; q < 8; q += 4) {
                float4* p = reinterpret_cast<float4*>(stage + Ly::K_BYTES + sw128b32_offset(t, j + q, kBT, 4));
                float4 r = *p;
                un[q] = r.x - xr[j + q];
                un[q + 1] = r.y - xr[j + q + 1];
                un[q + 2] = r.z - xr[j + q + 2];
                un[q + 3] = r.w - xr[j + q + 3];
                *reinterpret_cast<float4*>(vn + sw128_offset(t, j + q, kBT, 4)) =
                    make_float4(un[q], un[q + 1], un[q + 2], un[q + 3]);
                *p = make_float4(un[q] * dec, un[q + 1] * dec, un[q + 2] * dec, un[q + 3] * dec);
              }
            }
          }
        }
      }
    } else {
      // v tile <- v * exp(g_last - g_t)
      if (tid < kBT) sFac[tid] = __expf(gl - gc[tid]);
      __syncthreads();
      scale_rows<T>(stage + Ly::K_BYTES, kVT, sFac, tid, kThreads);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // U_c = k^T (scaled v / v_new) -- A = k^T (MN-major), B = v (MN-major)
    if (tid == 0) {
      if (MODE == 1 && (flags & kStoreVn)) {
#pragma unroll
        for (int j = 0; j < kVT / kBox; ++j)
          tma_store_3d(&tm_vn, sm + Ly::OFF_VN + j * kBT * 128, v0 + j * kBox, hh, row0);
      }
      if (MODE == 1) bulk_commit_group();
      tc_fence_after();
#pragma unroll
      for (int q = 0; q < kBT / kStep; ++q) {
        const uint32_t roff = q * kStep * 128;
        const uint64_t ad = make_sdesc(sk + roff, kBT * 128, kMNSbo, kMNLayout);
        const uint64_t bd = make_sdesc(sv + roff, kBT * 128, kMNSbo, kMNLayout);
        mma_kind<kBf16>(tU, ad, bd, kIdU, q > 0);
      }
      mma_commit(bar_mma);
    }
    pending = (int)mphase;
    ok = mbar_wait(bar_mma, mphase, &g_status_h);
    mphase ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    pending = -1;
    tc_fence_after();

    // Stage st is free: prefetch chunk c+2 (tiles by TMA, gates by cp.async).
    if (c + 2 < NT) {
      last_issued = c + 2;
      if (tid == 0) issue_tma(c + 2, st);
      if (tid < kBT) cp_async4(&sG[st * 64 + tid], g + (long long)(b * T_len + (c + 2) * kBT + tid) * H + hh);
    }
    cp_async_commit();

    // S = exp(g_last) S + U_c
    {
      float ur[kVT];
      tmem_ld64(tU + lane_off, ur);
      const float eg = __expf(gl);
      if (srow_ok) {
#pragma unroll
        for (int j = 0; j < kVT; j += 2) {
          const float2 r2 = __ffma2_rn(make_float2(eg, eg), make_float2(S[j], S[j + 1]), make_float2(ur[j], ur[j + 1]));
          S[j] = r2.x;
          S[j + 1] = r2.y;
        }
      }
    }
    tc_fence_before();
    if constexpr (MODE == 0) {
      // h[c] = state after chunk c, through the staging tile and a TMA store.
      if (tid == 0) bulk_wait_group_read0();
      __syncthreads();
      if (srow_ok) write_state_row<HT, false>(sm + Ly::OFF_HST, kk, K, S);
      fence_proxy_async_smem();
      __syncthreads();
      if (tid == 0) {
        store_h(c);
        bulk_commit_group();
      }
    }
  }
  cp_async_wait<0>();
  if (tid == 0) bulk_wait_group0();

  if (ok && MODE == 1 && final_state != nullptr && srow_ok) {
    float* dst = final_state + (((long long)b * H + hh) * K + kk) * V + v0;
#pragma unroll
    for (int j = 0; j < kVT; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
  }
  if (!ok) {
    // A wait ran out of time: one more bounded wait for what is in flight.
    if (pending >= 0) mbar_wait(bar_mma, (uint32_t)pending, &g_status_h);
    for (int j = consumed + 1; j <= last_issued; ++j) mbar_wait(&bar_tma[j & 1], (j >> 1) & 1, &g_status_h);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, Ly::TMEM_COLS);
}

template <typename T, int K, int MODE, bool HB>
int launch(const void* k, const void* w, const void* v, const float* g, const float* h0, void* h, void* v_new,
           float* final_state, int B, int T_len, int H, int V, cudaStream_t st) {
  using Ly = Layout<T, K, MODE, HB>;
  constexpr bool bf = Ly::BF16;
  const CUtensorMapDataType dt = bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const CUtensorMapSwizzle mn_sw = bf ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  const int es = sizeof(T);
  const int NT = T_len / kBT;
  const uint64_t rows = (uint64_t)B * T_len;
  const uint32_t box[3] = {(uint32_t)(128 / es), 1u, (uint32_t)kBT};
  CUtensorMap tk, tv, tw, th, tvn;
  {
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)H, rows};
    uint64_t str[2] = {(uint64_t)K * es, (uint64_t)H * K * es};
    int r = encode_tiled(&tk, dt, 3, k, dims, str, box, mn_sw);
    if (r == THM_OK && MODE == 1) r = encode_tiled(&tw, dt, 3, w, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (r != THM_OK) return r;
    if (MODE == 0) tw = tk;  // unused
  }
  {
    uint64_t dims[3] = {(uint64_t)V, (uint64_t)H, rows};
    uint64_t str[2] = {(uint64_t)V * es, (uint64_t)H * V * es};
    int r = encode_tiled(&tv, dt, 3, v, dims, str, box, mn_sw);
    if (r == THM_OK && MODE == 1 && v_new != nullptr)
      r = encode_tiled(&tvn, dt, 3, v_new, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    else
      tvn = tv;  // unused
    if (r != THM_OK) return r;
  }
  {
    // h [B*NT*H*K, V] as stored; the smem tile is either the state operand
    // (32-B atoms when fp32 activations) or the 16-B-chunk staging tile.
    const int hes = HB ? 2 : 4;
    uint64_t dims[2] = {(uint64_t)V, (uint64_t)B * NT * H * K};
    uint64_t str[1] = {(uint64_t)V * hes};
    uint32_t hbox[2] = {(uint32_t)(128 / hes), (uint32_t)K};
    const CUtensorMapSwizzle hsw = (Ly::H_FROM_S && !bf) ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
    int r = h != nullptr ? encode_tiled(&th, HB ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                                        2, h, dims, str, hbox, hsw)
                         : THM_OK;
    if (h == nullptr) th = tk;  // delta mode without the h output: no h store is issued
    if (r != THM_OK) return r;
  }
  auto kern = chunk_fwd_h_kernel<T, K, MODE, HB>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Ly::SMEM) != cudaSuccess)
    return THM_ERR_CUDA;
  dim3 grid(V / kVT, B * H);
  const int flags = (v_new != nullptr ? kStoreVn : 0) | (h != nullptr ? kStoreH : 0);
  kern<<<grid, kThreads, Ly::SMEM, st>>>(tk, tv, tw, th, tvn, g, h0, final_state, flags, T_len, H, V);
  return check_launch();
}

template <typename T, int MODE>
int dispatch_k(const void* k, const void* w, const void* v, const float* g, const float* h0, void* h, void* vn,
               float* fs, int B, int T_len, int H, int K, int V, bool hb, cudaStream_t st) {
  if (K == 64)
    return hb ? launch<T, 64, MODE, true>(k, w, v, g, h0, h, vn, fs, B, T_len, H, V, st)
              : launch<T, 64, MODE, false>(k, w, v, g, h0, h, vn, fs, B, T_len, H, V, st);
  return hb ? launch<T, 128, MODE, true>(k, w, v, g, h0, h, vn, fs, B, T_len, H, V, st)
            : launch<T, 128, MODE, false>(k, w, v, g, h0, h, vn, fs, B, T_len, H, V, st);
}

}  // namespace chunk_h
}  // namespace thm

THM_STATUS_READER(thm_internal_status_h, g_status_h)

extern "C" int thm_chunk_fwd_h_fwd(const void* k, const void* w, const void* v, const float* g, const float* h0,
                                   void* h, void* v_new, float* final_state, int B, int T, int H, int K, int V,
                                   int dtype, int h_dtype, int mode, thm_stream_t stream) {
  using namespace thm;
  if (B < 0 || T < 0 || H < 0 || K <= 0 || V <= 0 || T % 64 != 0) return THM_ERR_INVALID;
  if (dtype != THM_F32 && dtype != THM_BF16) return THM_ERR_INVALID;
  if (h_dtype != THM_F32 && h_dtype != THM_BF16) return THM_ERR_INVALID;
  if (mode != 0 && mode != 1) return THM_ERR_INVALID;
  if (mode == 0 && (w || h0 || v_new || final_state)) return THM_ERR_INVALID;
  if (mode == 1 && !w) return THM_ERR_INVALID;
  if ((long long)B * H == 0) return THM_OK;
  if (T == 0) {
    // No chunks: the final state is h0 (or zero).
    if (mode == 1 && final_state) {
      const size_t n = (size_t)B * H * K * V * sizeof(float);
      cudaError_t e = h0 ? cudaMemcpyAsync(final_state, h0, n, cudaMemcpyDeviceToDevice, (cudaStream_t)stream)
                         : cudaMemsetAsync(final_state, 0, n, (cudaStream_t)stream);
      return e == cudaSuccess ? THM_OK : THM_ERR_CUDA;
    }
    return THM_OK;
  }
  if (!k || !v || !g || (!h && mode == 0)) return THM_ERR_INVALID;
  if (!(K == 64 || K == 128) || !(V == 64 || V == 128)) return THM_ERR_UNSUPPORTED;
  if (!aligned16(k) || !aligned16(v) || (h && !aligned16(h)) || (w && !aligned16(w)) || (h0 && !aligned16(h0)) ||
      (v_new && !aligned16(v_new)) || (final_state && !aligned16(final_state)))
    return THM_ERR_ALIGNMENT;
  if ((long long)B * H > 65535) return THM_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool hb = h_dtype == THM_BF16;
  if (dtype == THM_BF16) {
    return mode == 0 ? chunk_h::dispatch_k<__nv_bfloat16, 0>(k, w, v, g, h0, h, v_new, final_state, B, T, H, K, V, hb, st)
                     : chunk_h::dispatch_k<__nv_bfloat16, 1>(k, w, v, g, h0, h, v_new, final_state, B, T, H, K, V, hb, st);
  }
  return mode == 0 ? chunk_h::dispatch_k<float, 0>(k, w, v, g, h0, h, v_new, final_state, B, T, H, K, V, hb, st)
                   : chunk_h::dispatch_k<float, 1>(k, w, v, g, h0, h, v_new, final_state, B, T, H, K, V, hb, st);
}
