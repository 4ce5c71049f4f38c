// gated_delta_ho.cu -- fused state recurrence and output of the gated delta
// rule: chunk_fwd_h (delta mode) and chunk_fwd_o in one pass over the chunks.
//
// The reference runs the two as separate kernels that meet in HBM
// (kernels/chunk_fwd_h/kernel.py:61-138 writes h, kernels/chunk_fwd_o/
// kernel.py:52-136 reads it back; docs/ARCHITECTURE.md:200-235 chains
// recompute_w_u -> chunk_fwd_h -> chunk_fwd_o). Here one CTA of 256 threads
// owns one (b, h) sequence (K = V = 128, bf16 activations) and walks its
// chunks in order; neither the per-chunk states h nor v_new ever reach HBM.
// Per chunk c, with the fp32 state h_c in registers (thread <-> row d of the
// state, one 64-column half per warpgroup) and a bf16 copy in shared memory:
//
//   S     = q k^T                           tcgen05 (M=64,  N=64,  K=128)
//   X     = w h_c,  G = q h_c               tcgen05 (M=64,  N=128, K=128)
//   P     = tril(S * e^{g_t - g_s})         TMEM -> registers -> smem (bf16)
//   v_new = u - X                            TMEM -> registers -> smem (bf16)
//   U     = k^T (v_new * e^{g_last - g_t})  tcgen05 (M=128, N=128, K=64)
//   L     = P v_new                          tcgen05 (M=64,  N=128, K=64)
//   h_{c+1} = e^{g_last} h_c + U             registers
//   o_c   = scale (L + e^{g_t} G)            registers -> smem -> TMA store
//
// The epilogue of chunk c-1 runs while the tensor core computes S, X, G of
// chunk c. Arithmetic matches the separate kernels of the chain: the state is
// rounded to bf16 only as an MMA operand (as the chain's bf16 h), v_new is
// rounded to bf16 once (as the chain's stored v_new).
//
// TMEM (512 columns): U [0,128) | X/G of chunk parity 0 [128,256) and 1
// [256,384) (X at lane 0, G at lane 16) | L [384,512) at lane 0, S [384,448)
// at lane 16. Shared memory: two 64 KB TMA stages (k, q, w, u tiles of a
// chunk, 128-B swizzle) + state copy 32 KB + v_new 16 KB + P 8 KB + o 16 KB.
#include <cuda_bf16.h>

#include "host_util.h"
#include "sm100.cuh"

THM_DEFINE_STATUS(g_status_ho)

namespace thm {
namespace delta_ho {

constexpr int kBT = 64;
constexpr int kK = 128;
constexpr int kV = 128;
constexpr int kMath = 256;             // math warps: 2 warpgroups
constexpr int kThreads = kMath + 64;   // + tcgen05 issuer warp + TMA producer warp
constexpr int kWG = kMath / 128;       // warps sharing a TMEM subpartition
constexpr int kCW = kV / kWG;          // V columns per math warp
constexpr int kPW = kBT / kWG;         // P columns per math warp

// 16x256b TMEM load of N/2 8-column groups (N = 2, 4 or 8 registers per group pair).
template <int N>
__device__ __forceinline__ void tmem_ld_16x256b(uint32_t taddr, float* v) {
  if constexpr (N == 8) tmem_ld_16x256b_x8(taddr, v);
  else if constexpr (N == 4) tmem_ld_16x256b_x4(taddr, v);
  else tmem_ld_16x256b_x2(taddr, v);
}

struct Layout {
  static constexpr int TILE = kBT * 128 * 2;  // [64 x 128] bf16 = two 8 KB boxes
  static constexpr int OFF_K = 0, OFF_Q = TILE, OFF_W = 2 * TILE, OFF_U = 3 * TILE;
  static constexpr int STAGE = 4 * TILE;                 // 64 KB
  static constexpr int OFF_S = 2 * STAGE;                // state copy [128 x 128] bf16, two 16 KB MN blocks
  static constexpr int OFF_VN = OFF_S + kK * kV * 2;     // v_new [64 x 128] bf16
  static constexpr int OFF_P = OFF_VN + TILE;            // P [64 x 64] bf16
  static constexpr int OFF_O = OFF_P + kBT * kBT * 2;    // o staging [64 x 128] bf16
  static constexpr int OFF_MISC = OFF_O + TILE;
  // misc: sG [2][64] | scale e^{g} [2][64] | barriers, TMEM slot
  static constexpr int SMEM = OFF_MISC + 2048 + 1024;
};

__device__ __forceinline__ uint32_t ld_u32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ float2 bf2_to_f2(uint32_t x) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x));
}

__global__ void __launch_bounds__(kThreads, 1)
    gated_delta_ho_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_q,
                          const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_u,
                          const __grid_constant__ CUtensorMap tm_o, const float* __restrict__ g,
                          const float* __restrict__ h0, float* __restrict__ final_state, float scale, int T_len,
                          int H) {
  using Ly = Layout;
  constexpr uint32_t kIdS = make_idesc(1u, 64, 64, 0, 0);
  constexpr uint32_t kIdXG = make_idesc(1u, 64, kV, 0, 1);
  constexpr uint32_t kIdU = make_idesc(1u, kK, kV, 1, 1);
  constexpr uint32_t kIdL = make_idesc(1u, 64, kV, 0, 1);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(sm);
  float* sG = reinterpret_cast<float*>(sm + Ly::OFF_MISC);           // [2][64]
  float* sEg = reinterpret_cast<float*>(sm + Ly::OFF_MISC + 512);    // [2][64] scale e^{g_t}
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Ly::OFF_MISC + 1024);
  uint64_t* full = bars;          // [2] TMA stage landed
  uint64_t* s_ready = bars + 2;   // h_c copied to smem (one arrival per math warp)
  uint64_t* vn_ready = bars + 3;  // v_new in smem (one arrival per math warp)
  uint64_t* p_ready = bars + 4;   // P in smem (one arrival per math warp)
  uint64_t* bar_s = bars + 5;     // S = q k^T in TMEM
  uint64_t* bar_a = bars + 6;     // X, G in TMEM
  uint64_t* bar_u = bars + 7;     // U in TMEM (stage consumed)
  uint64_t* bar_l = bars + 8;     // L in TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x;
  const int b = bh / H, hh = bh - (bh / H) * H;
  const int NT = T_len / kBT;

  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    mbar_init(s_ready, kMath / 32);
    mbar_init(vn_ready, kMath / 32);
    mbar_init(p_ready, kMath / 32);
    mbar_init(bar_s, 1);
    mbar_init(bar_a, 1);
    mbar_init(bar_u, 1);
    mbar_init(bar_l, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (tid < kBT) {
    sG[tid] = g[(long long)(b * T_len + tid) * H + hh];
    if (NT > 1) sG[64 + tid] = g[(long long)(b * T_len + kBT + tid) * H + hh];
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tU = tbase, tL = tbase + 384, tS = tbase + 384 + (16u << 16);
  bool ok = true;

  if (warp == kMath / 32 + 1) {
    // ---------------- TMA producer (one thread) ----------------
    if (lane == 0) {
      auto issue_tma = [&](int c) {
        const int st = c & 1;
        uint8_t* base = sm + st * Ly::STAGE;
        const int row0 = b * T_len + c * kBT;
        mbar_arrive_expect_tx(&full[st], Ly::STAGE);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          tma_load_3d(base + Ly::OFF_K + j * 8192, &tm_k, &full[st], j * 64, hh, row0);
          tma_load_3d(base + Ly::OFF_Q + j * 8192, &tm_q, &full[st], j * 64, hh, row0);
          tma_load_3d(base + Ly::OFF_W + j * 8192, &tm_w, &full[st], j * 64, hh, row0);
          tma_load_3d(base + Ly::OFF_U + j * 8192, &tm_u, &full[st], j * 64, hh, row0);
        }
      };
      issue_tma(0);
      if (NT > 1) issue_tma(1);
      int issued = NT > 1 ? 2 : 1;
      // Stage c & 1 is free once U(c) has read it.
      for (int c = 0; c + 2 < NT; ++c) {
        if (!mbar_wait(bar_u, c & 1, &g_status_ho)) { ok = false; break; }
        issue_tma(c + 2);
        issued = c + 3;
      }
      // No TMA may be in flight when the CTA exits: the last loads have landed (bounded).
      for (int j = issued - 2 < 0 ? 0 : issued - 2; j < issued; ++j) mbar_wait(&full[j & 1], (j >> 1) & 1, &g_status_ho);
    }
  } else if (warp == kMath / 32) {
    // ---------------- tcgen05 issuer (one thread) ----------------
    // Per chunk c: X, G | S of chunk c+1 (once P(c) has read S(c)) | U | L.
    if (lane == 0) {
      auto issue_s = [&](int c) {
        const uint32_t stg = sbase + (c & 1) * Ly::STAGE;
#pragma unroll
        for (int kq = 0; kq < kK / 16; ++kq) {
          const uint32_t off = (kq / 4) * 8192 + (kq % 4) * 32;
          mma_bf16_ss(tS, make_sdesc(stg + Ly::OFF_Q + off, 16, 1024), make_sdesc(stg + Ly::OFF_K + off, 16, 1024),
                      kIdS, kq > 0);
        }
        mma_commit(bar_s);
      };
      uint64_t* last_bar = nullptr;  // last commit, waited (bounded) before TMEM is released
      uint32_t last_ph = 0;
      if (mbar_wait(&full[0], 0, &g_status_ho)) {
        tc_fence_after();
        issue_s(0);
        last_bar = bar_s;
      } else {
        ok = false;
      }
      for (int c = 0; c < NT && ok; ++c) {
        const int st = c & 1;
        const uint32_t ph = c & 1;
        const uint32_t stg = sbase + st * Ly::STAGE;
        const uint32_t tXG = tbase + 128 + 128 * st;
        // X = w h_c, G = q h_c (stage c landed: S(c) was issued after its full wait)
        if (!mbar_wait(s_ready, ph, &g_status_ho)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kq = 0; kq < kK / 16; ++kq) {
          const uint32_t off = (kq / 4) * 8192 + (kq % 4) * 32;
          const uint64_t hd = make_sdesc(sbase + Ly::OFF_S + kq * 2048, kK * 128, 1024);
          mma_bf16_ss(tXG, make_sdesc(stg + Ly::OFF_W + off, 16, 1024), hd, kIdXG, kq > 0);
          mma_bf16_ss(tXG + (16u << 16), make_sdesc(stg + Ly::OFF_Q + off, 16, 1024), hd, kIdXG, kq > 0);
        }
        mma_commit(bar_a);
        last_bar = bar_a, last_ph = ph;
        // S of chunk c+1 while the math warps form v_new(c): tS is free once P(c) is in smem.
        if (!mbar_wait(p_ready, ph, &g_status_ho)) { ok = false; break; }
        if (c + 1 < NT) {
          if (!mbar_wait(&full[st ^ 1], ((c + 1) >> 1) & 1, &g_status_ho)) { ok = false; break; }
          tc_fence_after();
          issue_s(c + 1);
          last_bar = bar_s, last_ph = (c + 1) & 1;
        }
        // U = k^T (v_new e^{g_last - g_t}), then L = P v_new
        if (!mbar_wait(vn_ready, ph, &g_status_ho)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int q = 0; q < kBT / 16; ++q)
          mma_bf16_ss(tU, make_sdesc(stg + Ly::OFF_K + q * 2048, 8192, 1024),
                      make_sdesc(stg + Ly::OFF_U + q * 2048, 8192, 1024), kIdU, q > 0);
        mma_commit(bar_u);
#pragma unroll
        for (int q = 0; q < kBT / 16; ++q)
          mma_bf16_ss(tL, make_sdesc(sbase + Ly::OFF_P + q * 32, 16, 1024),
                      make_sdesc(sbase + Ly::OFF_VN + q * 2048, 8192, 1024), kIdL, q > 0);
        mma_commit(bar_l);
        last_bar = bar_l, last_ph = ph;
      }
      // Commits complete in issue order: the last one covers every MMA issued.
      if (last_bar != nullptr) mbar_wait(last_bar, last_ph, &g_status_ho);
    }
  } else {
    // ---------------- math warps ----------------
    // Warp w reads TMEM lanes 32 (w % 4) ..; the kWG warps of a subpartition
    // split the 128 V columns (and the 64 P columns) between them.
    const int sp = warp & 3;
    const int qc = kCW * (warp >> 2);  // first V column of this warp
    const int pc = kPW * (warp >> 2);  // first P column of this warp
    const int kk = tid & 127;          // state row (d) of this thread
    const uint32_t lane_row = (uint32_t)(32 * sp) << 16;
    const int r0 = 16 * sp + (lane >> 2), r1 = r0 + 8;  // 16x256b rows of M=64 accumulators
    const int c4 = 2 * (lane & 3);

    float S[kCW];
#pragma unroll
    for (int j = 0; j < kCW; ++j) S[j] = 0.f;
    if (h0 != nullptr) {
      const float* src = h0 + (((long long)b * H + hh) * kK + kk) * kV + qc;
#pragma unroll
      for (int j = 0; j < kCW; j += 4) {
        const float4 x = *reinterpret_cast<const float4*>(src + j);
        S[j] = x.x; S[j + 1] = x.y; S[j + 2] = x.z; S[j + 3] = x.w;
      }
    }

    // o tile of chunk j: scale L + scale e^{g_t} G -> staging -> TMA store.
    // Its first named barrier is also the uniform timeout vote.
    auto epilogue = [&](int j, bool good) -> bool {
      if (tid == 0) bulk_wait_group_read0();  // the previous o tile has left the staging buffer
      if (!named_bar_and(1, kMath, good)) return false;
      tc_fence_after();
      const float e0 = sEg[(j & 1) * 64 + r0], e1 = sEg[(j & 1) * 64 + r1];
      uint8_t* ob = sm + Ly::OFF_O;
#pragma unroll
      for (int hq = 0; hq < kCW / 32; ++hq) {  // 32 columns at a time (register pressure)
        float lv[16], gv[16];
        tmem_ld_16x256b_x4(tL + lane_row + qc + 32 * hq, lv);
        tmem_ld_16x256b_x4(tbase + 128 + 128 * (j & 1) + lane_row + (16u << 16) + qc + 32 * hq, gv);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int cc = qc + 32 * hq + 8 * q + c4;
          *reinterpret_cast<uint32_t*>(ob + sw128_offset(r0, cc, kBT, 2)) =
              pack_bf16x2(fmaf(lv[4 * q], scale, gv[4 * q] * e0), fmaf(lv[4 * q + 1], scale, gv[4 * q + 1] * e0));
          *reinterpret_cast<uint32_t*>(ob + sw128_offset(r1, cc, kBT, 2)) =
              pack_bf16x2(fmaf(lv[4 * q + 2], scale, gv[4 * q + 2] * e1), fmaf(lv[4 * q + 3], scale, gv[4 * q + 3] * e1));
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      named_bar_sync(1, kMath);
      if (tid == 0) {
        const int row0 = b * T_len + j * kBT;
        tma_store_3d(&tm_o, sm + Ly::OFF_O, 0, hh, row0);
        tma_store_3d(&tm_o, sm + Ly::OFF_O + 8192, 64, hh, row0);
        bulk_commit_group();
      }
      return true;
    };

    for (int c = 0; c < NT; ++c) {
      const int st = c & 1;
      const uint32_t ph = c & 1;
      uint8_t* stage = sm + st * Ly::STAGE;
      const float* gc = sG + st * 64;
      const uint32_t tXG = tbase + 128 + 128 * st;

      // (1) h_c -> shared memory (bf16, MN-major B operand of X and G)
      {
        uint8_t* tile = sm + Ly::OFF_S + (qc >> 6) * (kK * 128);
#pragma unroll
        for (int j = 0; j < kCW; j += 8) {
          uint4 p;
          p.x = pack_bf16x2(S[j], S[j + 1]);
          p.y = pack_bf16x2(S[j + 2], S[j + 3]);
          p.z = pack_bf16x2(S[j + 4], S[j + 5]);
          p.w = pack_bf16x2(S[j + 6], S[j + 7]);
          *reinterpret_cast<uint4*>(tile + sw128_offset(kk, (qc & 63) + j, kK, 2)) = p;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_ready);  // one arrival per warp

      // (2) epilogue of chunk c-1 while the tensor core computes X, G of chunk c
      cp_async_wait<0>();  // this chunk's gates have landed (visible after the next barrier)
      if (c > 0) {
        ok = mbar_wait(bar_l, (c - 1) & 1, &g_status_ho) && ok;
        if (!epilogue(c - 1, ok)) { ok = false; break; }
      } else if (!named_bar_and(1, kMath, ok)) {
        ok = false;
        break;
      }
      // Gates of chunk c+1 into sG[st^1]: every thread is past chunk c-1, its last reader.
      if (c >= 1 && c + 1 < NT && tid < kBT)
        cp_async4(&sG[(st ^ 1) * 64 + tid], g + (long long)(b * T_len + (c + 1) * kBT + tid) * H + hh);
      cp_async_commit();
      const float gl = gc[kBT - 1];
      const float g0 = gc[r0], g1 = gc[r1];
      if (tid < kBT) sEg[st * 64 + tid] = __expf(gc[tid]) * scale;

      // (3) P = tril(S e^{g_t - g_s}) -> smem (this warp: kPW columns), while X, G run
      ok = mbar_wait(bar_s, ph, &g_status_ho) && ok;
      tc_fence_after();
      {
        float sv[kPW / 2];
        tmem_ld_16x256b<kPW / 4>(tS + lane_row + pc, sv);
        uint8_t* pb = sm + Ly::OFF_P;
#pragma unroll
        for (int q = 0; q < kPW / 8; ++q) {
          const int cc = pc + 8 * q + c4;
          const float gc0 = gc[cc], gc1 = gc[cc + 1];
          const float p00 = (cc <= r0) ? sv[4 * q] * __expf(g0 - gc0) : 0.f;
          const float p01 = (cc + 1 <= r0) ? sv[4 * q + 1] * __expf(g0 - gc1) : 0.f;
          const float p10 = (cc <= r1) ? sv[4 * q + 2] * __expf(g1 - gc0) : 0.f;
          const float p11 = (cc + 1 <= r1) ? sv[4 * q + 3] * __expf(g1 - gc1) : 0.f;
          *reinterpret_cast<uint32_t*>(pb + sw128_offset(r0, cc, kBT, 2)) = pack_bf16x2(p00, p01);
          *reinterpret_cast<uint32_t*>(pb + sw128_offset(r1, cc, kBT, 2)) = pack_bf16x2(p10, p11);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_ready);  // one arrival per warp

      // (4) v_new = u - X -> smem (this warp: kCW columns)
      ok = mbar_wait(bar_a, ph, &g_status_ho) && ok;
      tc_fence_after();
      {
        float xv[kCW / 2];
        tmem_ld_16x256b<kCW / 8>(tXG + lane_row + qc, xv);
        const float d0 = __expf(gl - g0), d1 = __expf(gl - g1);
        uint8_t* ut = stage + Ly::OFF_U;
        uint8_t* vn = sm + Ly::OFF_VN;
#pragma unroll
        for (int q = 0; q < kCW / 8; ++q) {
          const int cc = qc + 8 * q + c4;
          const uint32_t o0 = sw128_offset(r0, cc, kBT, 2), o1 = sw128_offset(r1, cc, kBT, 2);
          const float2 u0 = bf2_to_f2(ld_u32(ut + o0)), u1 = bf2_to_f2(ld_u32(ut + o1));
          const float n00 = u0.x - xv[4 * q], n01 = u0.y - xv[4 * q + 1];
          const float n10 = u1.x - xv[4 * q + 2], n11 = u1.y - xv[4 * q + 3];
          // v_new (bf16, B operand of L) and v_new e^{g_last - g_t} (bf16, B operand
          // of U), each rounded once from the fp32 difference.
          *reinterpret_cast<uint32_t*>(vn + o0) = pack_bf16x2(n00, n01);
          *reinterpret_cast<uint32_t*>(vn + o1) = pack_bf16x2(n10, n11);
          *reinterpret_cast<uint32_t*>(ut + o0) = pack_bf16x2(n00 * d0, n01 * d0);
          *reinterpret_cast<uint32_t*>(ut + o1) = pack_bf16x2(n10 * d1, n11 * d1);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(vn_ready);  // one arrival per warp

      // (5) h_{c+1} = e^{g_last} h_c + U
      ok = mbar_wait(bar_u, ph, &g_status_ho) && ok;
      tc_fence_after();
      {
        const float eg = __expf(gl);
#pragma unroll
        for (int hq = 0; hq < kCW / 32; ++hq) {
          float ur[32];
          tmem_ld32(tU + lane_row + qc + 32 * hq, ur);
#pragma unroll
          for (int j = 0; j < 32; ++j) S[32 * hq + j] = fmaf(eg, S[32 * hq + j], ur[j]);
        }
      }
      tc_fence_before();
    }
    if (ok && NT > 0) ok = mbar_wait(bar_l, (NT - 1) & 1, &g_status_ho);
    if (ok && NT > 0) ok = epilogue(NT - 1, ok);
    cp_async_wait<0>();
    if (tid == 0) bulk_wait_group0();
    if (ok && final_state != nullptr) {
      float* dst = final_state + (((long long)b * H + hh) * kK + kk) * kV + qc;
#pragma unroll
      for (int j = 0; j < kCW; j += 4)
        *reinterpret_cast<float4*>(dst + j) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
    }
  }

  if (!ok) record_status(&g_status_ho, THM_ERR_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 512);
}

int launch(const void* q, const void* k, const void* w, const void* u, const float* g, const float* h0, void* o,
           float* final_state, float scale, int B, int T_len, int H, cudaStream_t st) {
  const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint64_t rows = (uint64_t)B * T_len;
  const uint32_t box[3] = {64u, 1u, (uint32_t)kBT};
  const uint64_t dims[3] = {128u, (uint64_t)H, rows};
  const uint64_t str[2] = {128u * 2, (uint64_t)H * 128 * 2};
  CUtensorMap tk, tq, tw, tu, to;
  int r = encode_tiled(&tk, dt, 3, k, dims, str, box);
  if (r == THM_OK) r = encode_tiled(&tq, dt, 3, q, dims, str, box);
  if (r == THM_OK) r = encode_tiled(&tw, dt, 3, w, dims, str, box);
  if (r == THM_OK) r = encode_tiled(&tu, dt, 3, u, dims, str, box);
  if (r == THM_OK) r = encode_tiled(&to, dt, 3, o, dims, str, box);
  if (r != THM_OK) return r;
  if (cudaFuncSetAttribute(gated_delta_ho_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Layout::SMEM) !=
      cudaSuccess)
    return THM_ERR_CUDA;
  gated_delta_ho_kernel<<<B * H, kThreads, Layout::SMEM, st>>>(tk, tq, tw, tu, to, g, h0, final_state, scale,
                                                                T_len, H);
  return check_launch();
}

}  // namespace delta_ho
}  // namespace thm

THM_STATUS_READER(thm_internal_status_ho, g_status_ho)

extern "C" int thm_gated_delta_fwd_ho(const void* q, const void* k, const void* w, const void* u, const float* g,
                                      const float* h0, void* o, float* final_state, float scale, int B, int T, int H,
                                      int K, int V, int dtype, thm_stream_t stream) {
  using namespace thm;
  if (B < 0 || T < 0 || H < 0 || K <= 0 || V <= 0 || T % 64 != 0) return THM_ERR_INVALID;
  if (dtype != THM_F32 && dtype != THM_BF16) return THM_ERR_INVALID;
  if ((long long)B * H == 0) return THM_OK;
  if (T == 0) {
    if (final_state) {
      const size_t n = (size_t)B * H * K * V * sizeof(float);
      cudaError_t e = h0 ? cudaMemcpyAsync(final_state, h0, n, cudaMemcpyDeviceToDevice, (cudaStream_t)stream)
                         : cudaMemsetAsync(final_state, 0, n, (cudaStream_t)stream);
      return e == cudaSuccess ? THM_OK : THM_ERR_CUDA;
    }
    return THM_OK;
  }
  if (!q || !k || !w || !u || !g || !o) return THM_ERR_INVALID;
  if (dtype != THM_BF16 || K != 128 || V != 128) return THM_ERR_UNSUPPORTED;
  if (!aligned16(q) || !aligned16(k) || !aligned16(w) || !aligned16(u) || !aligned16(o) || (h0 && !aligned16(h0)) ||
      (final_state && !aligned16(final_state)))
    return THM_ERR_ALIGNMENT;
  if ((long long)B * H > 0x7fffffffLL) return THM_ERR_UNSUPPORTED;
  return delta_ho::launch(q, k, w, u, g, h0, o, final_state, scale, B, T, H, reinterpret_cast<cudaStream_t>(stream));
}
