// gated_delta_ho.cu -- fused state recurrence and output of the gated delta
// rule: chunk_fwd_h (delta mode) and chunk_fwd_o in one pass over the chunks.
//
// The reference runs the two as separate kernels that meet in HBM
// (kernels/chunk_fwd_h/kernel.py:61-138 writes h, kernels/chunk_fwd_o/
// kernel.py:52-136 reads it back; docs/ARCHITECTURE.md:200-235 chains
// recompute_w_u -> chunk_fwd_h -> chunk_fwd_o). Here one CTA owns one (b, h)
// sequence (K = V = 128, bf16 activations) and walks its chunks in order;
// neither the per-chunk states h nor v_new ever reach HBM. Per chunk c, with
// the fp32 state h_c in registers (thread <-> state row d, one 64-column half
// per warpgroup) and a bf16 copy of it in shared memory:
//
//   [X; G] = [w; q] h_c                  tcgen05 M=128, N=128, K=128
//   [.; S] = [w; q] k^T                  tcgen05 M=128, N=64,  K=128 (rows 64..127)
//   v_new  = u - X                        rows t on TMEM lanes 0..63
//   V''    = v_new e^{g_last - g_t}       the B operand of U (and of L, below)
//   U      = k^T V''                      tcgen05 M=128, N=128, K=64
//   [X; D] += [0; P'] V''                 tcgen05 M=128, N=128, K=64, onto [X; G]
//   h_{c+1} = e^{g_last} h_c + U          registers
//   o_c    = scale e^{g_t} D              rows t on lanes 64..127 -> TMA store
//
// with P' = e^{-g_last} tril(S): then D = G + e^{-g_t} tril(S e^{g_t - g_s}) v_new, the
// causal term with its decay split into a column factor (folded into V'', which U needs
// anyway) and a row factor e^{-g_t} shared with G, so one fp32 scale per row recovers o
// without losing the smaller term. The v_new warps write one tile, P needs no
// exponentials, the epilogue reads one accumulator, and S needs no TMEM of L's (its
// product is issued right after [X; G] instead of after the previous epilogue). All
// factors stay within e^{60} while a chunk's gates span at most 60 and g_last >= -60
// ("plain" chunks, all of BASELINE's); another chunk ("steep") keeps the direct form:
// P = tril(S e^{g_t - g_s}), L = P v_new with v_new as its own tile, L in the columns it
// shares with S, o = scale (e^{g_t} G + L).
//
// w and q of a chunk sit in shared memory as one stacked [w; q] K-major tile,
// so X and G (and S) are single M=128 products: full-rate tensor-core shapes
// with half the instructions of two M=64 products, and the state copy is read
// once. With M=128 accumulators row t lives on TMEM lane t (X) or 64+t (G, S,
// L), so the math warps split by subpartition: the warps on lanes 0..63 form
// v_new (the state path) while the warps on lanes 64..127 write the previous
// chunk's output and form P. The state is carried in fp32 and rounded to bf16
// only as an MMA operand, v_new once to bf16 (its decayed copy).
//
// Shared memory carries about 330 KB per chunk (the operand reads of the four
// products, the TMA stage, the tiles the math warps write), some 1.3 us of its 128 B
// per clock: the v_new warps write one tile, not two.
//
// TMEM (512 columns): U [0,128) | [X; G] of chunk parity 0 [128,256) and 1
// [256,384) | S [384,448), sharing [384,512) with a steep chunk's L (S(c+1) waits
// until the epilogue has read that L). Shared memory: two 64 KB TMA stages (k, [w; q], u
// tiles of a chunk, 128-B swizzle) + state copy 32 KB + v_new 16 KB + [pad; P]
// 16 KB + o 16 KB.
#include <cuda_bf16.h>

#include "host_util.h"
#include "sm100.cuh"

THM_DEFINE_STATUS(g_status_ho)

namespace thm {
namespace delta_ho {

constexpr int kBT = 64;
constexpr int kK = 128;
constexpr int kV = 128;
constexpr int kMath = 256;            // 8 math warps: 4 on TMEM lanes 0..63, 4 on lanes 64..127
constexpr int kThreads = kMath + 64;  // + tcgen05 issuer warp + TMA producer warp
constexpr float kPlainSpan = 60.f;    // gate span up to which a chunk takes the one-tile form

struct Layout {
  static constexpr int TILE = kBT * 128 * 2;  // [64 x 128] bf16 = two 8 KB boxes
  static constexpr int OFF_K = 0;              // k: boxes j at +8 KB j
  static constexpr int OFF_WQ = TILE;          // [w; q]: K-block j at +16 KB j, w rows then q rows
  static constexpr int OFF_U = 3 * TILE;       // u: boxes j at +8 KB j
  static constexpr int STAGE = 4 * TILE;       // 64 KB
  static constexpr int OFF_S = 2 * STAGE;      // state copy [128 x 128] bf16, two 16 KB MN blocks
  static constexpr int OFF_VN = OFF_S + kK * kV * 2;  // v_new [64 x 128] bf16
  static constexpr int OFF_P = OFF_VN + TILE;         // [pad 8 KB; P [64 x 64] bf16]
  static constexpr int OFF_O = OFF_P + 2 * kBT * kBT * 2;  // o staging [64 x 128] bf16
  static constexpr int OFF_MISC = OFF_O + TILE;
  // misc: sG [3][64] | scale e^{g_t} [2][64] | e^{g_m - g_s} [64] | output factor of L [2][64] |
  //       plain-chunk flags [2] | barriers, TMEM slot
  static constexpr int SMEM = OFF_MISC + 2304 + 1024;
};

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
  constexpr uint32_t kIdXG = make_idesc(1u, 128, kV, 0, 1);
  constexpr uint32_t kIdS = make_idesc(1u, 128, 64, 0, 0);
  constexpr uint32_t kIdU = make_idesc(1u, kK, kV, 1, 1);
  constexpr uint32_t kIdL = make_idesc(1u, 128, kV, 0, 1);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(sm);
  float* sG = reinterpret_cast<float*>(sm + Ly::OFF_MISC);           // [3][64] gates, ring
  float* sEg = reinterpret_cast<float*>(sm + Ly::OFF_MISC + 768);    // [2][64] scale e^{g_t}
  float* sEb = reinterpret_cast<float*>(sm + Ly::OFF_MISC + 1280);   // [64] e^{g_m - g_s} of the chunk
  float* sEr = reinterpret_cast<float*>(sm + Ly::OFF_MISC + 1536);   // [2][64] factor of L in o
  int* sPlain = reinterpret_cast<int*>(sm + Ly::OFF_MISC + 2048);    // [2] chunk gates span <= kPlainSpan
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Ly::OFF_MISC + 2064);
  uint64_t* full = bars;          // [2] TMA stage landed
  uint64_t* s_ready = bars + 2;   // h_c copied to smem (one arrival per math warp)
  uint64_t* vn_ready = bars + 3;  // v_new in smem (one arrival per lane-0..63 warp)
  uint64_t* p_ready = bars + 4;   // P in smem (one arrival per lane-64..127 warp)
  uint64_t* e_done = bars + 5;    // L of the previous chunk read out (lane-64..127 warps)
  uint64_t* bar_s = bars + 6;     // S in TMEM
  uint64_t* bar_a = bars + 7;     // X, G in TMEM
  uint64_t* bar_u = bars + 8;     // U in TMEM (stage consumed)
  uint64_t* bar_l = bars + 9;     // L in TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x;
  const int b = bh / H, hh = bh - (bh / H) * H;
  const int NT = T_len / kBT;

  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    mbar_init(s_ready, kMath / 32);
    mbar_init(vn_ready, kMath / 64);
    mbar_init(p_ready, kMath / 64);
    mbar_init(e_done, kMath / 64);
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
  if (tid < kMath) {
    // rows 0..63 of the L product's A operand: never read back, zeroed so the
    // unused accumulator rows stay finite
    reinterpret_cast<uint4*>(sm + Ly::OFF_P)[2 * tid] = make_uint4(0, 0, 0, 0);
    reinterpret_cast<uint4*>(sm + Ly::OFF_P)[2 * tid + 1] = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tU = tbase, tL = tbase + 384, tS = tbase + 384;
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
          tma_load_3d(base + Ly::OFF_WQ + j * 16384, &tm_w, &full[st], j * 64, hh, row0);
          tma_load_3d(base + Ly::OFF_WQ + j * 16384 + 8192, &tm_q, &full[st], j * 64, hh, row0);
          tma_load_3d(base + Ly::OFF_U + j * 8192, &tm_u, &full[st], j * 64, hh, row0);
        }
      };
      issue_tma(0);
      if (NT > 1) issue_tma(1);
      int issued = NT > 1 ? 2 : 1;
      // Stage c & 1 is free once U(c) -- the last reader of k, w, q, u -- is done.
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
    // Per chunk c: [X; G] | S (after the epilogue has read L(c-1)) | U | L.
    if (lane == 0) {
      uint64_t* last_bar = nullptr;  // last commit, waited (bounded) before TMEM is released
      uint32_t last_ph = 0;
      for (int c = 0; c < NT && ok; ++c) {
        const int st = c & 1;
        const uint32_t ph = c & 1;
        const uint32_t stg = sbase + st * Ly::STAGE;
        const uint32_t tXG = tbase + 128 + 128 * st;
        // [X; G] = [w; q] h_c
        if (!mbar_wait(&full[st], (c >> 1) & 1, &g_status_ho) || !mbar_wait(s_ready, ph, &g_status_ho)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kq = 0; kq < kK / 16; ++kq)
          mma_bf16_ss(tXG, make_sdesc(stg + Ly::OFF_WQ + (kq / 4) * 16384 + (kq % 4) * 32, 16, 1024),
                      make_sdesc(sbase + Ly::OFF_S + kq * 2048, kK * 128, 1024), kIdXG, kq > 0);
        mma_commit(bar_a);
        last_bar = bar_a, last_ph = ph;
        // [.; S] = [w; q] k^T. Its columns double as a steep chunk's L: after a steep
        // chunk S waits until the epilogue has read that L.
        if (c > 0 && !sPlain[st ^ 1] && !mbar_wait(e_done, ph ^ 1, &g_status_ho)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kq = 0; kq < kK / 16; ++kq) {
          const uint32_t koff = (kq / 4) * 8192 + (kq % 4) * 32;
          mma_bf16_ss(tS, make_sdesc(stg + Ly::OFF_WQ + (kq / 4) * 16384 + (kq % 4) * 32, 16, 1024),
                      make_sdesc(stg + Ly::OFF_K + koff, 16, 1024), kIdS, kq > 0);
        }
        mma_commit(bar_s);
        last_bar = bar_s;
        // U = k^T (v_new e^{g_last - g_t}): the v_new tile of a plain chunk, else the
        // decayed copy the v_new warps wrote over u
        if (!mbar_wait(vn_ready, ph, &g_status_ho)) { ok = false; break; }
        tc_fence_after();
        const uint32_t vd = sPlain[st] ? sbase + Ly::OFF_VN : stg + Ly::OFF_U;
#pragma unroll
        for (int q = 0; q < kBT / 16; ++q)
          mma_bf16_ss(tU, make_sdesc(stg + Ly::OFF_K + q * 2048, 8192, 1024),
                      make_sdesc(vd + q * 2048, 8192, 1024), kIdU, q > 0);
        mma_commit(bar_u);
        last_bar = bar_u;
        // [.; L] = [pad; P] V: a plain chunk's L accumulates onto G in the [X; G] buffer
        // (the zero pad rows leave X as it is), a steep chunk's goes to its own columns
        if (!mbar_wait(p_ready, ph, &g_status_ho)) { ok = false; break; }
        tc_fence_after();
        const bool plain_c = sPlain[st] != 0;
        const uint32_t tLc = plain_c ? tXG : tL;
#pragma unroll
        for (int q = 0; q < kBT / 16; ++q)
          mma_bf16_ss(tLc, make_sdesc(sbase + Ly::OFF_P + q * 32, 16, 1024),
                      make_sdesc(sbase + Ly::OFF_VN + q * 2048, 8192, 1024), kIdL, plain_c || q > 0);
        mma_commit(bar_l);
        last_bar = bar_l;
      }
      // Commits complete in issue order: the last one covers every MMA issued.
      if (last_bar != nullptr) mbar_wait(last_bar, last_ph, &g_status_ho);
    }
  } else {
    // ---------------- math warps ----------------
    const int sp = warp & 3;          // TMEM subpartition: lanes 32 sp .. 32 sp + 31
    const int half = warp >> 2;       // 64-column half of V
    const int qc = 64 * half;
    const int kk = tid & 127;         // state row (d) of this thread
    const uint32_t lane_row = (uint32_t)(32 * sp) << 16;
    const bool xwarp = sp < 2;        // lanes 0..63: X rows; else G, S, L rows
    const int t = (32 * sp + lane) & 63;  // chunk row this thread reads from a M=128 accumulator
    const int gidx = xwarp ? -1 : ((half * 64) + (sp - 2) * 32 + lane);  // index among lane-64..127 warps

    float S[64];
#pragma unroll
    for (int j = 0; j < 64; ++j) S[j] = 0.f;
    if (h0 != nullptr) {
      const float* src = h0 + (((long long)b * H + hh) * kK + kk) * kV + qc;
#pragma unroll
      for (int j = 0; j < 64; j += 4) {
        const float4 x = *reinterpret_cast<const float4*>(src + j);
        S[j] = x.x; S[j + 1] = x.y; S[j + 2] = x.z; S[j + 3] = x.w;
      }
    }

    // o of chunk j (lane-64..127 warps): row t, this warp's 64 columns, staged in shared
    // memory and written by one TMA store (stores straight from registers would send 32
    // rows per warp instruction through the L1 pipeline the shared-memory traffic uses).
    // Plain chunk: the accumulator holds D = G + e^{-g_t} L, so o = scale e^{g_t} D;
    // steep chunk: o = scale (e^{g_t} G + L) from two accumulators.
    auto epilogue = [&](int j) {
      if (gidx == 0) bulk_wait_group_read0();  // the previous o tile has left the staging buffer
      named_bar_sync(3, kMath / 2);
      tc_fence_after();
      const bool plain_j = sPlain[j & 1] != 0;
      const float eg = sEg[(j & 1) * 64 + t];
      const float el = sEr[(j & 1) * 64 + t];
      const uint32_t tD = tbase + 128 + 128 * (j & 1) + lane_row + qc;
      uint8_t* ob = sm + Ly::OFF_O + half * 8192 + t * 128;
#pragma unroll
      for (int hq = 0; hq < 4; ++hq) {
        float gv[16], lv[16];
        tmem_ld16(tD + 16 * hq, gv);
        if (!plain_j) {
          tmem_ld16(tL + lane_row + qc + 16 * hq, lv);
        } else {
#pragma unroll
          for (int z = 0; z < 16; ++z) lv[z] = 0.f;
        }
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const float* l8 = lv + 8 * q;
          const float* g8 = gv + 8 * q;
          // el L + eg G, as packed fp32x2 (each lane an fmaf of the same operands)
          uint32_t w4[4];
#pragma unroll
          for (int z = 0; z < 4; ++z) {
            const float2 r2 = __ffma2_rn(make_float2(l8[2 * z], l8[2 * z + 1]), make_float2(el, el),
                                         __fmul2_rn(make_float2(g8[2 * z], g8[2 * z + 1]), make_float2(eg, eg)));
            w4[z] = pack_bf16x2(r2.x, r2.y);
          }
          *reinterpret_cast<uint4*>(ob + ((uint32_t)((2 * hq + q) ^ (t & 7)) << 4)) =
              make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(e_done);  // L(j) read: S of the next chunk may overwrite it
      named_bar_sync(3, kMath / 2);
      if (gidx == 0) {
        const int row0 = b * T_len + j * kBT;
        tma_store_3d(&tm_o, sm + Ly::OFF_O, 0, hh, row0);
        tma_store_3d(&tm_o, sm + Ly::OFF_O + 8192, 64, hh, row0);
        bulk_commit_group();
      }
    };

    for (int c = 0; c < NT; ++c) {
      const int st = c & 1;
      const uint32_t ph = c & 1;
      uint8_t* stage = sm + st * Ly::STAGE;
      const float* gc = sG + (c % 3) * 64;
      const uint32_t tXG = tbase + 128 + 128 * st;

      // (1) h_c -> shared memory (bf16, MN-major B operand of [X; G])
      {
        uint8_t* tile = sm + Ly::OFF_S + half * (kK * 128);
#pragma unroll
        for (int j = 0; j < 64; j += 8) {
          uint4 p;
          p.x = pack_bf16x2(S[j], S[j + 1]);
          p.y = pack_bf16x2(S[j + 2], S[j + 3]);
          p.z = pack_bf16x2(S[j + 4], S[j + 5]);
          p.w = pack_bf16x2(S[j + 6], S[j + 7]);
          *reinterpret_cast<uint4*>(tile + sw128_offset(kk, j, kK, 2)) = p;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_ready);

      const float gl = gc[kBT - 1];
      const float g_t = gc[t];
      // A chunk is "plain" when its gates span at most kPlainSpan: then both U and L
      // take the one tile v_new e^{g_last - g_s}, with L = tril(S) (v_new e^{g_last - g_s})
      // and o's factor e^{g_t - g_last} on L (both within e^{kPlainSpan}); otherwise v_new
      // and its decayed copy are separate tiles and P carries e^{g_t - g_s} itself.
      float gmn = fminf(gc[lane], gc[lane + 32]), gmx = fmaxf(gc[lane], gc[lane + 32]);
#pragma unroll
      for (int m = 16; m >= 1; m >>= 1) {
        gmn = fminf(gmn, __shfl_xor_sync(0xffffffffu, gmn, m));
        gmx = fmaxf(gmx, __shfl_xor_sync(0xffffffffu, gmx, m));
      }
      const bool plain = gmx - gmn <= kPlainSpan && gl >= -kPlainSpan;  // CTA-uniform
      if (xwarp) {
        // (2x) v_new = u - X for row t, this warp's 64 columns
        if (tid < kBT) {
          sEg[st * 64 + tid] = __expf(gc[tid]) * scale;
          sEr[st * 64 + tid] = scale;
        }
        if (tid == 0) sPlain[st] = plain ? 1 : 0;
        ok = mbar_wait(bar_a, ph, &g_status_ho) && ok;
        tc_fence_after();
        const float d = __expf(gl - g_t);
        const uint8_t* urow = stage + Ly::OFF_U + half * 8192 + t * 128;
        uint8_t* uw = stage + Ly::OFF_U + half * 8192 + t * 128;
        uint8_t* vrow = sm + Ly::OFF_VN + half * 8192 + t * 128;
#pragma unroll
        for (int hq = 0; hq < 2; ++hq) {
          float xv[32];
          tmem_ld32(tXG + lane_row + qc + 32 * hq, xv);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t off = (uint32_t)((4 * hq + q) ^ (t & 7)) << 4;
            const uint4 uu = *reinterpret_cast<const uint4*>(urow + off);
            const uint32_t uw4[4] = {uu.x, uu.y, uu.z, uu.w};
            uint32_t vn4[4], us4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 u2 = bf2_to_f2(uw4[e]);
              // u - x as fma(x, -1, u): the same rounding as the subtraction
              const float2 n = __ffma2_rn(make_float2(xv[8 * q + 2 * e], xv[8 * q + 2 * e + 1]),
                                          make_float2(-1.f, -1.f), u2);
              // v_new e^{g_last - g_t} (B operand of U; of L too for a plain chunk) and,
              // for a steep chunk, v_new itself (B operand of L), each rounded to bf16 once
              // from the fp32 difference.
              vn4[e] = pack_bf16x2(n.x, n.y);
              const float2 nd = __fmul2_rn(n, make_float2(d, d));
              us4[e] = pack_bf16x2(nd.x, nd.y);
            }
            if (plain) {
              *reinterpret_cast<uint4*>(vrow + off) = make_uint4(us4[0], us4[1], us4[2], us4[3]);
            } else {
              *reinterpret_cast<uint4*>(vrow + off) = make_uint4(vn4[0], vn4[1], vn4[2], vn4[3]);
              *reinterpret_cast<uint4*>(uw + off) = make_uint4(us4[0], us4[1], us4[2], us4[3]);
            }
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(vn_ready);
      } else {
        // (2g) epilogue of chunk c-1, then P(c) = tril(S e^{g_t - g_s}) for row t
        if (c > 0) {
          ok = mbar_wait(bar_l, (c - 1) & 1, &g_status_ho) && ok;
          epilogue(c - 1);
        }
        // Steep chunk: the decay e^{g_t - g_s} = e^{g_t - g_m} e^{g_m - g_s} about the middle
        // g_m of the chunk's gate range: 64 + 1 exponentials per chunk instead of one per
        // entry. Each factor is at most e^{range / 2}; chunks whose gates span more than 120
        // (factors past e^60) take one exponential per entry instead.
        const bool factored = gmx - gmn <= 120.f;  // CTA-uniform
        const float gm = 0.5f * (gmn + gmx);
        float a_t = 1.f;
        const float eml = __expf(-gl);  // plain chunk: P' = e^{-g_last} tril(S)
        if (!plain) {
          if (gidx < kBT) sEb[gidx] = __expf(gm - gc[gidx]);
          named_bar_sync(3, kMath / 2);
          a_t = __expf(g_t - gm);
        }
        ok = mbar_wait(bar_s, ph, &g_status_ho) && ok;
        tc_fence_after();
        uint8_t* prow = sm + Ly::OFF_P + 8192 + t * 128;
        if (half == 1 && t < 32) {
          // columns 32..63 of rows 0..31 are above the diagonal
#pragma unroll
          for (int q = 4; q < 8; ++q) *reinterpret_cast<uint4*>(prow + ((uint32_t)(q ^ (t & 7)) << 4)) = make_uint4(0, 0, 0, 0);
        } else {
          float sv[32];
          tmem_ld32(tS + lane_row + 32 * half, sv);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t p4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int s0 = 32 * half + 8 * q + 2 * e;
              float2 f;
              if (plain) {
                f = make_float2(eml, eml);
              } else if (factored) {
                f = __fmul2_rn(make_float2(a_t, a_t), make_float2(sEb[s0], sEb[s0 + 1]));
              } else {
                f = make_float2(__expf(g_t - gc[s0]), __expf(g_t - gc[s0 + 1]));
              }
              const float2 pr = __fmul2_rn(make_float2(sv[8 * q + 2 * e], sv[8 * q + 2 * e + 1]), f);
              p4[e] = pack_bf16x2((s0 <= t) ? pr.x : 0.f, (s0 + 1 <= t) ? pr.y : 0.f);
            }
            *reinterpret_cast<uint4*>(prow + ((uint32_t)((4 * half + q) ^ (t & 7)) << 4)) =
                make_uint4(p4[0], p4[1], p4[2], p4[3]);
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_ready);
      }

      // (3) h_{c+1} = e^{g_last} h_c + U; all math threads vote (uniform timeout exit)
      ok = mbar_wait(bar_u, ph, &g_status_ho) && ok;
      cp_async_wait<0>();  // gates of chunk c+1 (issued one iteration ago) have landed
      if (!named_bar_and(1, kMath, ok)) { ok = false; break; }
      // Gates of chunk c+2 into ring slot (c+2) % 3: its last readers (chunk c-1) are done.
      if (c + 2 < NT && tid < kBT)
        cp_async4(&sG[((c + 2) % 3) * 64 + tid], g + (long long)(b * T_len + (c + 2) * kBT + tid) * H + hh);
      cp_async_commit();
      tc_fence_after();
      {
        const float eg = __expf(gl);
#pragma unroll
        for (int hq = 0; hq < 2; ++hq) {
          float ur[32];
          tmem_ld32(tU + lane_row + qc + 32 * hq, ur);
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float2 r2 = __ffma2_rn(make_float2(eg, eg), make_float2(S[32 * hq + j], S[32 * hq + j + 1]),
                                         make_float2(ur[j], ur[j + 1]));
            S[32 * hq + j] = r2.x;
            S[32 * hq + j + 1] = r2.y;
          }
        }
      }
      tc_fence_before();
    }
    if (ok && NT > 0 && !xwarp) {
      ok = mbar_wait(bar_l, (NT - 1) & 1, &g_status_ho);
      epilogue(NT - 1);
    }
    cp_async_wait<0>();
    if (gidx == 0) bulk_wait_group0();
    if (ok && final_state != nullptr) {
      float* dst = final_state + (((long long)b * H + hh) * kK + kk) * kV + qc;
#pragma unroll
      for (int j = 0; j < 64; j += 4)
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
