// Pass-1 score kernels of the two-pass sparse decode and the score-key packer.
//
// Follows src/attention_kernels.py of the reference (saifmb0/bytes):
//   sparse_score_scalar  (:1077-1133)  scores = scaling * q.k over bf16 / fp8 keys
//   sparse_score_packed  (:1136-1222)  k = code*scale + zero from uint8-packed 2/4-bit
//                                      keys, per-token groups of `group_size` channels
//   quantize_and_pack_score_keys (:1225-1249)
// Output scores [B,Hq,S] fp32.
//
// Design: one CTA per (batch, KV head, head chunk, token split); K tiles stream into
// shared memory (cp.async, 3 stages); all G query heads of the KV head are scored from
// the same tile on the tensor cores (S^T[16 tok x 8 heads] = K . Q^T, mma.sync). Packed
// codes are unpacked in registers as exact f16 subnormals (code*2^-24): one shift and one
// AND give two MMA operands. Per-token scale/zero enter in fp32 after the contraction:
// score = sum_g s_g * (sum_{c in g} q_c code_c) + z_g * (sum_{c in g} q_c).
#include "common.cuh"
#include "decode_shared.cuh"

#include <algorithm>
#include <cmath>

namespace bd {
namespace {

constexpr int kSW = 4;         // warps per CTA
constexpr int kSStages = 3;
// packed keys (2/4 bits): the per-token unpack -> MMA chain needs more warps in flight than
// the bf16/fp8 forms, so their tiles double-buffer and four CTAs share an SM (at 4 bits and
// group size 32, 48 KB of double-buffered tiles; smaller groups fit three)
__host__ __device__ constexpr bool packed_kt(int kt) { return kt == 2 || kt == 4; }
__host__ __device__ constexpr int score_stages(int kt) { return packed_kt(kt) ? 2 : kSStages; }
__host__ __device__ constexpr int score_ctas_per_sm(int kt) { return packed_kt(kt) ? 4 : 2; }
constexpr float kSub = 16777216.f;

// KT: 16 = bf16 keys, 8 = fp8 keys, 4 / 2 = packed bits; GS: group size of packed keys
template <int KT, int D, int GS>
struct SL {
  static constexpr int RB = KT == 16 ? 1 : (KT == 8 ? 2 : 4);  // 16-token row blocks per warp per tile
  static constexpr int TILE = 16 * kSW * RB;
  static constexpr int ROWB = KT == 16 ? D * 2 : (KT == 8 ? D : D * KT / 8);
  // packed rows are read by 8 lanes at a time with 16-byte loads: pitches chosen conflict-free
  static constexpr int PITCH = (KT == 16 || KT == 8) ? ROWB + 16 : (ROWB == 16 ? 16 : (ROWB == 32 ? 48 : 80));
  static constexpr int KBYTES = TILE * PITCH;
  static constexpr int SZB = (KT == 16 || KT == 8) ? 0 : TILE * (D / GS) * 2;  // scale (zero) tile: D/GS f16 per token
  static constexpr int STAGE = KBYTES + 2 * SZB;
};

struct ScoreParams {
  const void* q; int64_t q_sb, q_sh; int q_dtype;
  const uint8_t* k; int64_t k_sb, k_sh, k_ss;  // strides in elements of k's dtype (bytes for packed/fp8)
  const uint16_t* sc; int64_t sc_sb, sc_sh, sc_ss;  // scale (bf16/f16 bits) [B,Hk,S,D/gs]
  const uint16_t* zr; int64_t zr_sb, zr_sh, zr_ss;
  int sz_bf16;
  int gs;  // group size (packed only)
  float* out; int64_t o_sb, o_sh;
  int B, Hq, Hk, G, S;
  int head_chunks, heads_per_chunk, tiles_per_split;
  float scaling;
};

__device__ __forceinline__ float load_qs(const ScoreParams& p, int64_t off) {
  switch (p.q_dtype) {
    case BD_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.q)[off]);
    case BD_F16: return __half2float(reinterpret_cast<const __half*>(p.q)[off]);
    default: return reinterpret_cast<const float*>(p.q)[off];
  }
}
__device__ __forceinline__ float h16_to_f(uint16_t u, int is_bf16) {
  return is_bf16 ? __uint_as_float(uint32_t(u) << 16) : __half2float(__ushort_as_half(u));
}
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
// N consecutive 16-bit floats (bf16 or f16) from shared memory, one vector load (2N bytes,
// 2N-byte aligned), widened to fp32
template <int N>
__device__ __forceinline__ void load_row16(const uint16_t* src, int is_bf16, float* out) {
  uint32_t w[(N + 1) / 2];
  if constexpr (N == 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(src);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (N == 4) {
    const uint2 v = *reinterpret_cast<const uint2*>(src);
    w[0] = v.x; w[1] = v.y;
  } else if constexpr (N == 2) {
    w[0] = *reinterpret_cast<const uint32_t*>(src);
  } else {
    w[0] = *src;
  }
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const uint32_t h = (w[i >> 1] >> (16 * (i & 1))) & 0xffffu;
    out[i] = h16_to_f(uint16_t(h), is_bf16);
  }
}

// GS: group size of packed keys (compile-time, so every per-group accumulator index is
// static and the accumulators stay in registers); 0 for bf16 / fp8 keys.
template <int KT, int D, int NT, int GS>
__global__ void __launch_bounds__(kSW * 32, score_ctas_per_sm(KT)) score_kernel(const ScoreParams p) {
  griddep_wait();  // programmatic launch: the previous kernel's results are complete past here
  griddep_launch_dependents();
  using L = SL<KT, D, GS>;
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int KSTEPS = D / 16;
  constexpr int NGMAX = GS > 0 ? D / GS : 1;  // groups per token row
  static_assert(KT == 16 || KT == 8 || (GS >= 16 && D % GS == 0), "packed keys need a group size");
  const int split = blockIdx.x;
  const int hk = blockIdx.y / p.head_chunks;
  const int chunk = blockIdx.y % p.head_chunks;
  const int b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int t_begin = split * p.tiles_per_split * L::TILE;
  const int t_end = min(p.S, t_begin + p.tiles_per_split * L::TILE);
  const int ntiles = t_end > t_begin ? (t_end - t_begin + L::TILE - 1) / L::TILE : 0;
  const int h0 = chunk * p.heads_per_chunk;
  const int nheads = min(p.heads_per_chunk, p.G - h0);
  const uint8_t* kbase = p.k + (int64_t(b) * p.k_sb + int64_t(hk) * p.k_sh) * (KT == 16 ? 2 : 1);

  // ---- B fragments (query), channel order depends on the key layout
  uint32_t qb[KSTEPS][NT][2];
  float score_mul = p.scaling;
  float qsum[NGMAX][NT][2];  // packed keys: per-group sum of the f16 query, heads 2tq,2tq+1
  {
    float qv[KSTEPS][NT][4];
    float amax = 0.f;
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int hl = nt * 8 + g;
        const bool ok = hl < nheads;
        const int64_t qoff = int64_t(b) * p.q_sb + int64_t(hk * p.G + h0 + (ok ? hl : 0)) * p.q_sh;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          int c;
          if (KT == 16) c = kk * 16 + 2 * tq + (e & 1) + (e >> 1) * 8;  // ldmatrix order
          else if (KT == 8) c = kk * 16 + 4 * tq + e;                    // fp8 byte order
          else if (KT == 2) c = kk * 16 + tq + 8 * (e & 1) + 4 * (e >> 1);  // fields tq, tq+8 | tq+4, tq+12
          else c = kk * 16 + tq + 4 * (e & 1) + 8 * (e >> 1);             // fields tq, tq+4 | 8+tq, 12+tq
          qv[kk][nt][e] = ok ? load_qs(p, qoff + c) : 0.f;
          amax = fmaxf(amax, fabsf(qv[kk][nt][e]));
        }
      }
    float qs = 1.f;
    if (KT != 16) {
      amax = warp_max(amax);
      int ex = 0;
      frexpf(amax, &ex);
      const int shift = ex > 14 ? ex - 14 : 0;
      qs = ldexpf(1.f, -shift);
      score_mul = ldexpf(p.scaling, shift);
    }
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        if (KT == 16) {
          qb[kk][nt][0] = pack_bf16x2(qv[kk][nt][0], qv[kk][nt][1]);
          qb[kk][nt][1] = pack_bf16x2(qv[kk][nt][2], qv[kk][nt][3]);
        } else {
          qb[kk][nt][0] = pack_f16x2(qv[kk][nt][0] * qs, qv[kk][nt][1] * qs);
          qb[kk][nt][1] = pack_f16x2(qv[kk][nt][2] * qs, qv[kk][nt][3] * qs);
        }
      }
    if (KT == 2 || KT == 4) {
      // per-group sums of the f16 query for heads 2tq, 2tq+1: lane (g,tq) sums its 4
      // channels of head g per k-step, reduce over tq, then fetch heads 2tq(+1).
      float part[KSTEPS][NT];
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float2 a = __half22float2(*reinterpret_cast<__half2*>(&qb[kk][nt][0]));
          const float2 c = __half22float2(*reinterpret_cast<__half2*>(&qb[kk][nt][1]));
          float v = (a.x + a.y) + (c.x + c.y);
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          part[kk][nt] = v;  // sum over the 16 channels of k-step kk, head g (+nt*8)
        }
      constexpr int kpg = GS > 0 ? GS / 16 : 1;  // k-steps per group
#pragma unroll
      for (int gi = 0; gi < NGMAX; ++gi)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float v = 0.f;
#pragma unroll
          for (int kk = 0; kk < KSTEPS; ++kk)
            if (kk / kpg == gi) v += part[kk][nt];
          // 2^-24: the epilogue applies the subnormal codes' 2^24 to the whole score
          qsum[gi][nt][0] = __shfl_sync(0xffffffffu, v, (2 * tq) * 4) * (1.f / kSub);
          qsum[gi][nt][1] = __shfl_sync(0xffffffffu, v, (2 * tq + 1) * 4) * (1.f / kSub);
        }
      score_mul *= kSub;
      if (KT == 2) {
        // the operand registers of k-slots 2tq+8, 2tq+9 keep their codes 8 bits up (an exact
        // subnormal 2^8 larger, one mask instead of a shift and a mask): their query halves
        // are scaled by 2^-8 to match
        const __half2 sc8 = __float2half2_rn(1.f / 256.f);
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            qb[kk][nt][1] = h2_bits(__hmul2(bits_h2(qb[kk][nt][1]), sc8));
      }
    }
  }

  constexpr int ngroups = (KT == 2 || KT == 4) ? NGMAX : 0;
  const uint8_t* scb = (KT == 2 || KT == 4)
      ? reinterpret_cast<const uint8_t*>(p.sc + int64_t(b) * p.sc_sb + int64_t(hk) * p.sc_sh) : nullptr;
  const uint8_t* zrb = (KT == 2 || KT == 4)
      ? reinterpret_cast<const uint8_t*>(p.zr + int64_t(b) * p.zr_sb + int64_t(hk) * p.zr_sh) : nullptr;
  auto load_tile = [&](int tile, int stage) {
    const int t0 = t_begin + tile * L::TILE;
    const uint32_t ks = smem_u32(smem + stage * L::STAGE);
    constexpr int CH = L::ROWB / 16;
    for (int c = threadIdx.x; c < L::TILE * CH; c += kSW * 32) {
      const int r = c / CH, cc = c % CH;
      const int t = t0 + r;
      const bool ok = t < t_end;
      const int64_t rowoff = int64_t(ok ? t : t_begin) * p.k_ss * (KT == 16 ? 2 : 1);
      cp_async16(ks + r * L::PITCH + cc * 16, kbase + rowoff + cc * 16, ok ? 16 : 0);
    }
    if (KT == 2 || KT == 4) {
      // scale / zero rows of this tile are one contiguous block (token-major, ngroups f16 each)
      const int bytes_tile = L::TILE * ngroups * 2;
      const int64_t off0 = int64_t(t0) * ngroups * 2;
      const int64_t lim = int64_t(t_end) * ngroups * 2;
      for (int c = threadIdx.x; c < bytes_tile / 16; c += kSW * 32) {
        const int64_t off = off0 + c * 16;
        const int64_t rem = lim - off;
        const int valid = rem <= 0 ? 0 : (rem >= 16 ? 16 : int(rem));
        cp_async16(ks + L::KBYTES + c * 16, scb + (valid ? off : 0), valid);
        cp_async16(ks + L::KBYTES + L::SZB + c * 16, zrb + (valid ? off : 0), valid);
      }
    }
  };

  constexpr int NST = score_stages(KT);
#pragma unroll
  for (int s = 0; s < NST - 1; ++s) {
    if (s < ntiles) load_tile(s, s);
    cp_async_commit();
  }

  for (int it = 0; it < ntiles; ++it) {
    cp_async_wait<NST - 2>();
    __syncthreads();
    {
      const int nxt = it + NST - 1;
      if (nxt < ntiles) load_tile(nxt, nxt % NST);
      cp_async_commit();
    }
    const uint8_t* st = smem + (it % NST) * L::STAGE;
    const uint32_t ks = smem_u32(st);
    const uint16_t* ssc = reinterpret_cast<const uint16_t*>(st + L::KBYTES);
    const uint16_t* szr = reinterpret_cast<const uint16_t*>(st + L::KBYTES + L::SZB);
#pragma unroll
    for (int rb = 0; rb < L::RB; ++rb) {
      const int r0 = (warp * L::RB + rb) * 16;  // tile-local first row
      const int t0 = t_begin + it * L::TILE + r0;
      if (t0 >= t_end) break;
      float acc[NGMAX][NT][4];
#pragma unroll
      for (int gi = 0; gi < NGMAX; ++gi)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) acc[gi][nt][0] = acc[gi][nt][1] = acc[gi][nt][2] = acc[gi][nt][3] = 0.f;
      if (KT == 16) {
        const int arow = r0 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk) {
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4(a0, a1, a2, a3, ks + arow * L::PITCH + (kk * 16 + (lane >> 4) * 8) * 2);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma_bf16(acc[0][nt], a0, a1, a2, a3, qb[kk][nt][0], qb[kk][nt][1]);
        }
      } else if (KT == 8) {
        const int arow = r0 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
        for (int k2 = 0; k2 < KSTEPS / 2; ++k2) {
          uint32_t r0_, r1_, r2_, r3_;
          ldmatrix_x4(r0_, r1_, r2_, r3_, ks + arow * L::PITCH + k2 * 32 + (lane >> 4) * 16);
          const uint32_t x0 = e4m3x2_to_f16x2(r0_), x1 = e4m3x2_to_f16x2(r1_);
          const uint32_t x2 = e4m3x2_to_f16x2(r0_ >> 16), x3 = e4m3x2_to_f16x2(r1_ >> 16);
          const uint32_t y0 = e4m3x2_to_f16x2(r2_), y1 = e4m3x2_to_f16x2(r3_);
          const uint32_t y2 = e4m3x2_to_f16x2(r2_ >> 16), y3 = e4m3x2_to_f16x2(r3_ >> 16);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            mma_f16(acc[0][nt], x0, x1, x2, x3, qb[2 * k2][nt][0], qb[2 * k2][nt][1]);
            mma_f16(acc[0][nt], y0, y1, y2, y3, qb[2 * k2 + 1][nt][0], qb[2 * k2 + 1][nt][1]);
          }
        }
      } else {
        // packed codes: token rows g and g+8 of the row block
        constexpr int WPR = L::ROWB / 4;  // words per token row
        uint32_t wa[WPR], wb[WPR];
#pragma unroll
        for (int w4 = 0; w4 < WPR / 4; ++w4) {
          const uint4 x = *reinterpret_cast<const uint4*>(st + (r0 + g) * L::PITCH + w4 * 16);
          const uint4 y = *reinterpret_cast<const uint4*>(st + (r0 + g + 8) * L::PITCH + w4 * 16);
          wa[4 * w4] = x.x; wa[4 * w4 + 1] = x.y; wa[4 * w4 + 2] = x.z; wa[4 * w4 + 3] = x.w;
          wb[4 * w4] = y.x; wb[4 * w4 + 1] = y.y; wb[4 * w4 + 2] = y.z; wb[4 * w4 + 3] = y.w;
        }
        constexpr int kpg = GS > 0 ? GS / 16 : 1;
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk) {
          uint32_t a0, a1, a2, a3;
          if (KT == 2) {
            const uint32_t xa = wa[kk] >> (2 * tq), xb = wb[kk] >> (2 * tq);
            a0 = xa & 0x00030003u;
            a1 = xb & 0x00030003u;
            a2 = xa & 0x03000300u;  // code * 2^(8-24): see the query halves' 2^-8
            a3 = xb & 0x03000300u;
          } else {
            a0 = (wa[2 * kk] >> (4 * tq)) & 0x000F000Fu;
            a1 = (wb[2 * kk] >> (4 * tq)) & 0x000F000Fu;
            a2 = (wa[2 * kk + 1] >> (4 * tq)) & 0x000F000Fu;
            a3 = (wb[2 * kk + 1] >> (4 * tq)) & 0x000F000Fu;
          }
#pragma unroll
          for (int gi = 0; gi < NGMAX; ++gi)
            if (kk / kpg == gi)
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) mma_f16(acc[gi][nt], a0, a1, a2, a3, qb[kk][nt][0], qb[kk][nt][1]);
        }
      }
      // ---- epilogue: scale/zero, write scores
      const int ta = t0 + g, tb2 = t0 + g + 8;
      float res[NT][4];
      if (KT == 16 || KT == 8) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) res[nt][e] = acc[0][nt][e] * score_mul;
      } else {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) res[nt][0] = res[nt][1] = res[nt][2] = res[nt][3] = 0.f;
        // this token's NGMAX scales (zeros) are one 2*NGMAX-byte row of the tile
        const int la = r0 + g, lb = r0 + g + 8;  // tile-local rows (zero-filled past the end)
        float sa[NGMAX], za[NGMAX], sb[NGMAX], zb[NGMAX];
        load_row16<NGMAX>(ssc + la * NGMAX, p.sz_bf16, sa);
        load_row16<NGMAX>(szr + la * NGMAX, p.sz_bf16, za);
        load_row16<NGMAX>(ssc + lb * NGMAX, p.sz_bf16, sb);
        load_row16<NGMAX>(szr + lb * NGMAX, p.sz_bf16, zb);
#pragma unroll
        for (int gi = 0; gi < NGMAX; ++gi)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              res[nt][j] = fmaf(qsum[gi][nt][j], za[gi], fmaf(acc[gi][nt][j], sa[gi], res[nt][j]));
              res[nt][2 + j] = fmaf(qsum[gi][nt][j], zb[gi], fmaf(acc[gi][nt][2 + j], sb[gi], res[nt][2 + j]));
            }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) res[nt][e] *= score_mul;
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int hl = nt * 8 + 2 * tq + j;
          if (hl >= nheads) continue;
          float* orow = p.out + int64_t(b) * p.o_sb + int64_t(hk * p.G + h0 + hl) * p.o_sh;
          if (ta < t_end) orow[ta] = res[nt][j];
          if (tb2 < t_end) orow[tb2] = res[nt][2 + j];
        }
    }
  }
}

template <int KT, int D, int NT, int GS>
int launch_score(const ScoreParams& p, int n_splits, cudaStream_t st) {
  using L = SL<KT, D, GS>;
  const size_t smem = size_t(score_stages(KT)) * L::STAGE;
  auto kern = score_kernel<KT, D, NT, GS>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    int rc = cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
                        "cudaFuncSetAttribute(score)");
    if (rc) return rc;
    attr[dev & 63] = true;
  }
  dim3 grid(n_splits, p.Hk * p.head_chunks, p.B);
  return launch_programmatic(kern, grid, dim3(kSW * 32), smem, st, p, "score_kernel launch");
}

template <int KT, int D, int GS>
int launch_score_gs(const ScoreParams& p, int nt, int n_splits, cudaStream_t st) {
  return nt == 1 ? launch_score<KT, D, 1, GS>(p, n_splits, st) : launch_score<KT, D, 2, GS>(p, n_splits, st);
}

template <int KT, int D>
int launch_score_nt(const ScoreParams& p, int nt, int n_splits, cudaStream_t st) {
  if constexpr (KT == 16 || KT == 8) {
    return launch_score_gs<KT, D, 0>(p, nt, n_splits, st);
  } else {
    switch (p.gs) {
      case 16: return launch_score_gs<KT, D, 16>(p, nt, n_splits, st);
      case 32: return launch_score_gs<KT, D, 32>(p, nt, n_splits, st);
      case 64: return launch_score_gs<KT, D, 64>(p, nt, n_splits, st);
      default: return launch_score_gs<KT, D, (D >= 128 ? 128 : 64)>(p, nt, n_splits, st);
    }
  }
}

int tile_tokens(int kt) { return 16 * kSW * (kt == 16 ? 1 : (kt == 8 ? 2 : 4)); }

// ------------------------------------------------------------ full-precision scores
// CUDA-core fp32 form of the same scores for the inputs the tensor-core tiles would have
// to round: an fp32 query (the MMA operands are bf16 / f16), an f16 query against bf16
// keys, and f16 / fp32 keys. Every key element is widened to fp32 (packed codes
// dequantised as code * scale + zero, the reference's per-element form,
// src/attention_kernels.py:1175-1190); score = scaling * sum_d q_d * k_d, like the
// reference's fp32 Triton blocks (:1098-1110, :1169-1196) up to summation order.
// One CTA: 64 tokens of one (batch, KV head), the group's heads 16 at a time; the key tile
// sits in shared memory with a padded pitch (conflict-free column reads), each thread owns
// one token and 8 heads.
enum GenericKey { kGkBf16 = 0, kGkF16, kGkF32, kGkFp8, kGkPack4, kGkPack2 };
constexpr int kGenTok = 64;

template <int KIND, int D>
__global__ void __launch_bounds__(128) score_generic_kernel(const ScoreParams p) {
  __shared__ float ks[kGenTok][D + 1];
  __shared__ float qs[16][D];
  const int t0 = blockIdx.x * kGenTok, hk = blockIdx.y, b = blockIdx.z;
  const int nt = min(kGenTok, p.S - t0);
  for (int i = threadIdx.x; i < kGenTok * D; i += 128) {
    const int t = i / D, d = i % D;
    float x = 0.f;
    if (t < nt) {
      const int64_t tok = int64_t(b) * p.k_sb + int64_t(hk) * p.k_sh + int64_t(t0 + t) * p.k_ss;
      if (KIND == kGkBf16) x = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.k)[tok + d]);
      else if (KIND == kGkF16) x = __half2float(reinterpret_cast<const __half*>(p.k)[tok + d]);
      else if (KIND == kGkF32) x = reinterpret_cast<const float*>(p.k)[tok + d];
      else if (KIND == kGkFp8) x = float(reinterpret_cast<const __nv_fp8_e4m3*>(p.k)[tok + d]);
      else {
        constexpr int BITS = KIND == kGkPack4 ? 4 : 2, EPB = 8 / BITS;
        const uint32_t code = (uint32_t(p.k[tok + d / EPB]) >> ((d % EPB) * BITS)) & ((1u << BITS) - 1);
        const int g = d / p.gs;
        const float sc = h16_to_f(p.sc[int64_t(b) * p.sc_sb + int64_t(hk) * p.sc_sh + int64_t(t0 + t) * p.sc_ss + g], p.sz_bf16);
        const float zr = h16_to_f(p.zr[int64_t(b) * p.zr_sb + int64_t(hk) * p.zr_sh + int64_t(t0 + t) * p.zr_ss + g], p.sz_bf16);
        x = fmaf(float(code), sc, zr);
      }
    }
    ks[t][d] = x;
  }
  const int t = threadIdx.x % kGenTok, hsel = threadIdx.x / kGenTok;  // 2 head lanes
  for (int h0 = 0; h0 < p.G; h0 += 16) {
    const int nh = min(16, p.G - h0);
    __syncthreads();  // the key tile is written / the previous head chunk's readers are done
    for (int i = threadIdx.x; i < nh * D; i += 128) {
      const int h = i / D, d = i % D;
      qs[h][d] = load_qs(p, int64_t(b) * p.q_sb + int64_t(hk * p.G + h0 + h) * p.q_sh + d);
    }
    __syncthreads();
    if (t >= nt) continue;
    for (int h = hsel; h < nh; h += 2) {
      float acc = 0.f;
#pragma unroll 8
      for (int d = 0; d < D; ++d) acc = fmaf(qs[h][d], ks[t][d], acc);
      p.out[int64_t(b) * p.o_sb + int64_t(hk * p.G + h0 + h) * p.o_sh + t0 + t] = acc * p.scaling;
    }
  }
}

template <int D>
int launch_score_generic(const ScoreParams& p, int kind, cudaStream_t st) {
  dim3 grid(unsigned((p.S + kGenTok - 1) / kGenTok), unsigned(p.Hk), unsigned(p.B));
  switch (kind) {
    case kGkBf16: score_generic_kernel<kGkBf16, D><<<grid, 128, 0, st>>>(p); break;
    case kGkF16: score_generic_kernel<kGkF16, D><<<grid, 128, 0, st>>>(p); break;
    case kGkF32: score_generic_kernel<kGkF32, D><<<grid, 128, 0, st>>>(p); break;
    case kGkFp8: score_generic_kernel<kGkFp8, D><<<grid, 128, 0, st>>>(p); break;
    case kGkPack4: score_generic_kernel<kGkPack4, D><<<grid, 128, 0, st>>>(p); break;
    default: score_generic_kernel<kGkPack2, D><<<grid, 128, 0, st>>>(p); break;
  }
  return cuda_check(cudaGetLastError(), "score_generic_kernel launch");
}

// ------------------------------------------------------------ score-key pack
template <typename T, int BITS>
__global__ void pack_score_keys_kernel(const T* __restrict__ k, int64_t rows, int64_t r_h, int64_t s_b, int64_t s_h,
                                       int64_t s_s, int S, int D, int gs, uint8_t* __restrict__ packed,
                                       T* __restrict__ scale, T* __restrict__ zero) {
  const int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int ng = D / gs;
  if (gid >= rows * ng) return;
  const int64_t row = gid / ng;  // (b, h, s) flattened
  const int grp = int(gid % ng);
  const int64_t sidx = row % S, bh = row / S;
  const int64_t h = bh % r_h, bb = bh / r_h;
  const T* src = k + bb * s_b + h * s_h + sidx * s_s + int64_t(grp) * gs;
  float lo = INFINITY, hi = -INFINITY;
  for (int e = 0; e < gs; ++e) {
    const float x = to_f32<T>(src[e]);
    lo = fminf(lo, x);
    hi = fmaxf(hi, x);
  }
  constexpr int LV = (1 << BITS) - 1;
  // (max-min)/(levels-1) as PyTorch forms it on a CUDA device: times the fp32 reciprocal
  constexpr float kRcp = 1.0f / float(LV);
  const float sc = __fmul_rn(fmaxf(__fsub_rn(hi, lo), 1e-8f), kRcp);
  constexpr int EPB = 8 / BITS;
  uint8_t* dst = packed + row * (D / EPB) + int64_t(grp) * (gs / EPB);
  for (int e0 = 0; e0 < gs; e0 += EPB) {
    uint32_t byte = 0;
#pragma unroll
    for (int i = 0; i < EPB; ++i) {
      float qv = rintf(__fdiv_rn(__fsub_rn(to_f32<T>(src[e0 + i]), lo), sc));
      qv = fminf(fmaxf(qv, 0.f), float(LV));
      byte |= uint32_t(qv) << (i * BITS);
    }
    dst[e0 / EPB] = uint8_t(byte);
  }
  scale[row * ng + grp] = from_f32<T>(sc);
  zero[row * ng + grp] = from_f32<T>(lo);
}

}  // namespace
}  // namespace bd

extern "C" {

int bd_sparse_score(const bd_tensor* q, const bd_tensor* k, const bd_tensor* scale, const bd_tensor* zero,
                    float scaling, int score_bits, int group_size, const bd_tensor* scores, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if ((rc = check_tensor(q, "q", 3)) || (rc = check_tensor(k, "k", 4)) ||
      (rc = check_tensor(scores, "scores", 3, BD_F32)))
    return rc;
  if (q->dtype != BD_BF16 && q->dtype != BD_F16 && q->dtype != BD_F32) return fail(BD_ERR_DTYPE, "q must be bf16/f16/f32");
  const int64_t B = q->shape[0], Hq = q->shape[1], D = q->shape[2];
  const int64_t Hk = k->shape[1], S = k->shape[2];
  if (k->shape[0] != B || Hk <= 0 || Hq % Hk) return fail(BD_ERR_SHAPE, "k must be [B,Hk,S,*] with Hq % Hk == 0");
  if (D != 32 && D != 64 && D != 128) return fail(BD_ERR_UNSUPPORTED, "head_dim must be 32, 64 or 128");
  int kt;
  if (score_bits == 16) {
    if ((k->dtype != BD_BF16 && k->dtype != BD_F16 && k->dtype != BD_F32) || k->shape[3] != D)
      return fail(BD_ERR_DTYPE, "score_bits=16 needs bf16, f16 or f32 k [B,Hk,S,D]");
    kt = 16;
  } else if (score_bits == 8) {
    if (k->dtype != BD_F8E4M3 || k->shape[3] != D) return fail(BD_ERR_DTYPE, "score_bits=8 needs fp8 e4m3 k [B,Hk,S,D]");
    kt = 8;
  } else if (score_bits == 4 || score_bits == 2) {
    if (k->dtype != BD_U8 || k->shape[3] * (8 / score_bits) != D)
      return fail(BD_ERR_SHAPE, "packed k must be uint8 [B,Hk,S,D*bits/8]");
    if (group_size != 16 && group_size != 32 && group_size != 64 && group_size != 128)
      return fail(BD_ERR_UNSUPPORTED, "group_size must be 16, 32, 64 or 128");
    if (D % group_size) return fail(BD_ERR_SHAPE, "head_dim must be a multiple of group_size");
    if ((rc = check_tensor(scale, "scale", 4)) || (rc = check_tensor(zero, "zero", 4))) return rc;
    if (scale->dtype != zero->dtype || (scale->dtype != BD_BF16 && scale->dtype != BD_F16))
      return fail(BD_ERR_DTYPE, "scale/zero must both be bf16 or both f16");
    for (const bd_tensor* t : {scale, zero})
      if (t->shape[0] != B || t->shape[1] != Hk || t->shape[2] != S || t->shape[3] != D / group_size)
        return fail(BD_ERR_SHAPE, "scale/zero must be [B,Hk,S,D/group_size]");
    for (const bd_tensor* t : {scale, zero}) {
      const int64_t ng = D / group_size;
      if ((t->stride[3] != 1 && ng > 1) || (t->stride[2] != ng && S > 1))
        return fail(BD_ERR_STRIDE, "scale/zero must be token-major contiguous within each (batch, head)");
      if (reinterpret_cast<uintptr_t>(t->data) % 16 || (t->shape[1] > 1 && (t->stride[1] * 2) % 16) ||
          (t->shape[0] > 1 && (t->stride[0] * 2) % 16))
        return fail(BD_ERR_ALIGN, "scale/zero (batch, head) blocks must start on 16-byte boundaries");
    }
    kt = score_bits;
  } else {
    return fail(BD_ERR_VALUE, "Unsupported score_bits");
  }
  if (scores->shape[0] != B || scores->shape[1] != Hq || scores->shape[2] != S || (scores->stride[2] != 1 && S > 1))
    return fail(BD_ERR_SHAPE, "scores must be [B,Hq,S] with contiguous rows");
  if (q->stride[2] != 1) return fail(BD_ERR_STRIDE, "q innermost dim must be contiguous");
  if ((rc = check_rows_aligned(k, "k"))) return rc;
  if (B * Hq * S == 0) return BD_OK;
  ScoreParams p{};
  p.q = q->data; p.q_sb = q->stride[0]; p.q_sh = q->stride[1]; p.q_dtype = q->dtype;
  p.k = static_cast<const uint8_t*>(k->data); p.k_sb = k->stride[0]; p.k_sh = k->stride[1]; p.k_ss = k->stride[2];
  if (kt == 2 || kt == 4) {
    p.sc = static_cast<const uint16_t*>(scale->data); p.sc_sb = scale->stride[0]; p.sc_sh = scale->stride[1]; p.sc_ss = scale->stride[2];
    p.zr = static_cast<const uint16_t*>(zero->data); p.zr_sb = zero->stride[0]; p.zr_sh = zero->stride[1]; p.zr_ss = zero->stride[2];
    p.sz_bf16 = scale->dtype == BD_BF16;
    p.gs = group_size;
  }
  p.out = static_cast<float*>(scores->data); p.o_sb = scores->stride[0]; p.o_sh = scores->stride[1];
  p.B = int(B); p.Hq = int(Hq); p.Hk = int(Hk); p.G = int(Hq / Hk); p.S = int(S);
  const int nt = p.G <= 8 ? 1 : 2;
  p.heads_per_chunk = 8 * nt;
  p.head_chunks = (p.G + p.heads_per_chunk - 1) / p.heads_per_chunk;
  p.scaling = scaling;
  // inputs the tensor-core operands would round (fp32 query; f16 query against bf16 keys;
  // f16 / fp32 keys) take the fp32 CUDA-core kernel
  // (and head_dim 32, which the tensor-core tiles do not cover)
  const bool generic =
      D == 32 || q->dtype == BD_F32 || (kt == 16 && (k->dtype != BD_BF16 || q->dtype != BD_BF16));
  if (generic) {
    const int kind = kt == 16 ? (k->dtype == BD_BF16 ? kGkBf16 : k->dtype == BD_F16 ? kGkF16 : kGkF32)
                              : kt == 8 ? kGkFp8 : kt == 4 ? kGkPack4 : kGkPack2;
    cudaStream_t gst = reinterpret_cast<cudaStream_t>(stream);
    return D == 128 ? launch_score_generic<128>(p, kind, gst)
                    : D == 64 ? launch_score_generic<64>(p, kind, gst) : launch_score_generic<32>(p, kind, gst);
  }
  const int64_t tt = tile_tokens(kt);
  const int64_t ntiles = (S + tt - 1) / tt;
  const int64_t pairs = B * Hk * p.head_chunks;
  const int64_t slots = int64_t(score_ctas_per_sm(kt)) * num_sms();
  int64_t splits = pairs >= slots ? 1 : slots / pairs;
  splits = std::max<int64_t>(1, std::min<int64_t>(splits, ntiles));
  const int64_t tps = (ntiles + splits - 1) / splits;
  splits = (ntiles + tps - 1) / tps;
  p.tiles_per_split = int(tps);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int ns = int(splits);
  if (D == 128) {
    switch (kt) {
      case 16: return launch_score_nt<16, 128>(p, nt, ns, st);
      case 8: return launch_score_nt<8, 128>(p, nt, ns, st);
      case 4: return launch_score_nt<4, 128>(p, nt, ns, st);
      default: return launch_score_nt<2, 128>(p, nt, ns, st);
    }
  }
  switch (kt) {
    case 16: return launch_score_nt<16, 64>(p, nt, ns, st);
    case 8: return launch_score_nt<8, 64>(p, nt, ns, st);
    case 4: return launch_score_nt<4, 64>(p, nt, ns, st);
    default: return launch_score_nt<2, 64>(p, nt, ns, st);
  }
}

int bd_pack_score_keys(const bd_tensor* k, int score_bits, int group_size, const bd_tensor* packed,
                       const bd_tensor* scale, const bd_tensor* zero, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if (score_bits != 2 && score_bits != 4) return fail(BD_ERR_VALUE, "Unsupported score_bits");
  if ((rc = check_tensor(k, "k", 4)) || (rc = check_tensor(packed, "packed", 4, BD_U8)) ||
      (rc = check_tensor(scale, "scale", 4, k->dtype)) || (rc = check_tensor(zero, "zero", 4, k->dtype)))
    return rc;
  if (k->dtype != BD_BF16 && k->dtype != BD_F16 && k->dtype != BD_F32) return fail(BD_ERR_DTYPE, "k must be bf16/f16/f32");
  const int64_t B = k->shape[0], H = k->shape[1], S = k->shape[2], D = k->shape[3];
  if (group_size <= 0 || D % group_size || group_size % (8 / score_bits))
    return fail(BD_ERR_SHAPE, "head_dim must be a multiple of group_size");
  const int epb = 8 / score_bits;
  const int64_t ng = D / group_size;
  if (packed->shape[0] != B || packed->shape[1] != H || packed->shape[2] != S || packed->shape[3] != D / epb)
    return fail(BD_ERR_SHAPE, "packed must be [B,H,S,D*bits/8]");
  for (const bd_tensor* t : {scale, zero})
    if (t->shape[0] != B || t->shape[1] != H || t->shape[2] != S || t->shape[3] != ng)
      return fail(BD_ERR_SHAPE, "scale/zero must be [B,H,S,D/group_size]");
  auto dense = [](const bd_tensor* t) {
    int64_t s = 1;
    for (int i = 3; i >= 0; --i) {
      if (t->shape[i] > 1 && t->stride[i] != s) return false;
      s *= t->shape[i];
    }
    return true;
  };
  if (!dense(packed) || !dense(scale) || !dense(zero)) return fail(BD_ERR_STRIDE, "outputs must be contiguous");
  if (k->stride[3] != 1 && D > 1) return fail(BD_ERR_STRIDE, "k innermost dim must be contiguous");
  const int64_t rows = B * H * S;
  if (rows * D == 0) return BD_OK;
  const int64_t total = rows * ng;
  const unsigned blocks = unsigned((total + 127) / 128);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define BD_PSK(T)                                                                                                  \
  if (score_bits == 2)                                                                                             \
    pack_score_keys_kernel<T, 2><<<blocks, 128, 0, st>>>(static_cast<const T*>(k->data), rows, H, k->stride[0],    \
        k->stride[1], k->stride[2], int(S), int(D), group_size, static_cast<uint8_t*>(packed->data),               \
        static_cast<T*>(scale->data), static_cast<T*>(zero->data));                                                \
  else                                                                                                             \
    pack_score_keys_kernel<T, 4><<<blocks, 128, 0, st>>>(static_cast<const T*>(k->data), rows, H, k->stride[0],    \
        k->stride[1], k->stride[2], int(S), int(D), group_size, static_cast<uint8_t*>(packed->data),               \
        static_cast<T*>(scale->data), static_cast<T*>(zero->data));
  if (k->dtype == BD_BF16) { BD_PSK(__nv_bfloat16) }
  else if (k->dtype == BD_F16) { BD_PSK(__half) }
  else { BD_PSK(float) }
#undef BD_PSK
  return cuda_check(cudaGetLastError(), "pack_score_keys_kernel launch");
}

}  // extern "C"
