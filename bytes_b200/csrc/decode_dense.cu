// Dense GQA decode attention over a bf16 or fp8-e4m3 KV cache (split-KV flash-decoding).
//
// Follows decode_attn_bf16 / decode_attn_fp8 (src/attention_kernels.py:8-182 of the
// reference): per query head, softmax(scaling * q.k) . v with fp32 accumulation.
//
// Design (one CTA = one (batch, KV head, query-head chunk, key split)):
//  * 4 consumer warps; a 64-token tile is split into 16-token row blocks, one per warp.
//  * K/V tiles stream HBM -> shared memory through a 3-stage cp.async pipeline; the rows
//    land with a 16-byte pad so ldmatrix reads are bank-conflict free.
//  * The GQA group makes QK^T a dense contraction: S^T[16 tokens x 8 heads] =
//    K[16 x D] . Q^T[D x 8] on the tensor cores (mma.sync m16n8k16, bf16 or f16 in,
//    fp32 accumulate). Every K/V byte is read from HBM once per KV head, not G times.
//  * Online softmax in exp2 space on the accumulator fragments, its reference moved
//    lazily; P is transposed in registers (movmatrix) into the B operand of
//    O^T[D x 8] += V^T[D x 16] . P^T[16 x 8].
//  * Warps merge through shared memory; splits merge in a log-sum-exp combine kernel.
// fp8 keys/values are widened to f16 (exact) in registers; the query is fed as f16,
// pre-scaled by a power of two when its magnitude would exceed the f16 range.
#include "common.cuh"
#include "decode_shared.cuh"

#include <algorithm>
#include <cmath>
#include <mutex>

namespace bd {

namespace {

constexpr int kWarps = 4;
constexpr int kRows = 16 * kWarps;  // tokens per tile
constexpr int kStages = 3;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
// log2 headroom of the lazily moved softmax reference. Zero: the reference is the running
// maximum as in plain online softmax (the largest weight of a tile that moved it is exactly
// 1, which keeps bf16 P exact there); only the rescale is skipped when no score passes it.
constexpr float kHeadroomD = 0.f;

struct DenseParams {
  const void* q; int64_t q_sb, q_sh; int q_dtype;
  const uint8_t* k; int64_t k_sb, k_sh, k_ss;  // strides in elements
  const uint8_t* v; int64_t v_sb, v_sh, v_ss;
  int B, Hq, Hk, G, S;
  int head_chunks, heads_per_chunk;
  int tiles_per_split, n_splits;
  int split_offset, split_stride;  // partial index = (b*Hq+hq)*split_stride + split_offset + split
  float scale_log2;
  // split partials: index ((b*Hq + hq) * n_splits + split)
  float* part_m; float* part_l; float* part_o;
  // direct output when n_splits == 1 and final
  void* out; int out_dtype; int64_t o_sb, o_sh;
  int direct;
  // 1: launched as a programmatic dependent of the kernel before it in the stream, which
  // it does not read from; it waits for that kernel only before exiting, so a kernel
  // that waits on this one also sees the earlier kernel's writes.
  int pdl;
  // 1 (with pdl, one split): after that wait, merge partial slots [0, split_offset) of each
  // row with this CTA's own result and write `out`
  int merge;
  int smem_bytes;  // dynamic shared memory of the launch (the merge stages the slot rows there)
};

// merge-mode bulk copies whose barrier wait ran past its limit (a result is then wrong)
__device__ unsigned int g_merge_timeouts = 0;

template <typename T>
__device__ __forceinline__ float ldq(const void* base, int64_t off) {
  return to_f32<T>(reinterpret_cast<const T*>(base)[off]);
}

__device__ __forceinline__ float load_q(const DenseParams& p, int64_t off) {
  switch (p.q_dtype) {
    case BD_BF16: return ldq<__nv_bfloat16>(p.q, off);
    case BD_F16: return ldq<__half>(p.q, off);
    default: return ldq<float>(p.q, off);
  }
}

__device__ __forceinline__ void store_out(void* base, int dt, int64_t off, float x) {
  switch (dt) {
    case BD_BF16: reinterpret_cast<__nv_bfloat16*>(base)[off] = __float2bfloat16_rn(x); break;
    case BD_F16: reinterpret_cast<__half*>(base)[off] = __float2half_rn(x); break;
    default: reinterpret_cast<float*>(base)[off] = x; break;
  }
}

// CTAs per SM the split plan fills: fp8 tiles take half the shared memory of bf16 ones,
// and a third CTA hides more of each tile's convert -> MMA chain (32K, B = 8: 59.6 -> 58.0 us;
// four measured 60.1)
__host__ __device__ constexpr int dense_ctas_per_sm(bool fp8) { return fp8 ? 3 : 2; }

template <int D, int NT, bool FP8>
__global__ void __launch_bounds__(kWarps * 32, dense_ctas_per_sm(FP8)) dense_decode_kernel(const DenseParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  // a programmatic dependent queued behind this grid (the combine) may start launching;
  // it waits for this grid before reading anything
  griddep_launch_dependents();
  constexpr int ELT = FP8 ? 1 : 2;
  constexpr int ROWB = D * ELT;
  constexpr int PITCH = ROWB + 16;
  constexpr int TILEB = kRows * PITCH;
  constexpr int CHUNKS = ROWB / 16;
  constexpr int KSTEPS = D / 16;
  constexpr int NH = 8 * NT;  // heads per CTA (padded)

  const int split = blockIdx.x;
  const int hk = blockIdx.y / p.head_chunks;
  const int chunk = blockIdx.y % p.head_chunks;
  const int b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;

  const int t_begin = split * p.tiles_per_split * kRows;
  const int t_end = min(p.S, t_begin + p.tiles_per_split * kRows);
  const int ntiles = t_end > t_begin ? (t_end - t_begin + kRows - 1) / kRows : 0;
  const int h0 = chunk * p.heads_per_chunk;  // first local head of this chunk
  const int nheads = min(p.heads_per_chunk, p.G - h0);

  const uint8_t* kbase = p.k + (int64_t(b) * p.k_sb + int64_t(hk) * p.k_sh) * ELT;
  const uint8_t* vbase = p.v + (int64_t(b) * p.v_sb + int64_t(hk) * p.v_sh) * ELT;

  auto load_tile = [&](int tile, int stage) {
    const int t0 = t_begin + tile * kRows;
    const uint32_t ks = smem_u32(smem + stage * 2 * TILEB);
    const uint32_t vs = ks + TILEB;
    for (int c = threadIdx.x; c < kRows * CHUNKS; c += kWarps * 32) {
      const int r = c / CHUNKS, cc = c % CHUNKS;
      const int t = t0 + r;
      const bool ok = t < t_end;
      const int tt = ok ? t : t_begin;
      cp_async16(ks + r * PITCH + cc * 16, kbase + int64_t(tt) * p.k_ss * ELT + cc * 16, ok ? 16 : 0);
      cp_async16(vs + r * PITCH + cc * 16, vbase + int64_t(tt) * p.v_ss * ELT + cc * 16, ok ? 16 : 0);
    }
  };

  // first tiles in flight before the query loads, so the two latencies overlap
#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < ntiles) load_tile(s, s);
    cp_async_commit();
  }

  // ---- query fragments (B operand of QK^T), kept in registers for the whole split
  uint32_t qb[KSTEPS][NT][2];
  float score_mul = p.scale_log2;
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
          // bf16 path: natural channel order (2tq, 2tq+1, 2tq+8, 2tq+9);
          // fp8 path: the ldmatrix byte layout gives channels 4tq..4tq+3 per k-step.
          const int c = FP8 ? kk * 16 + 4 * tq + e : kk * 16 + 2 * tq + (e & 1) + (e >> 1) * 8;
          qv[kk][nt][e] = ok ? load_q(p, qoff + c) : 0.f;
          amax = fmaxf(amax, fabsf(qv[kk][nt][e]));
        }
      }
    float qscale = 1.f;
    if (FP8) {
      amax = warp_max(amax);
      // keep |q| below 2^15 in f16; power-of-two scaling is exact
      int ex = 0;
      frexpf(amax, &ex);
      const int shift = ex > 15 ? ex - 15 : 0;
      qscale = ldexpf(1.f, -shift);
      score_mul = ldexpf(p.scale_log2, shift);
    }
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        if (FP8) {
          qb[kk][nt][0] = pack_f16x2(qv[kk][nt][0] * qscale, qv[kk][nt][1] * qscale);
          qb[kk][nt][1] = pack_f16x2(qv[kk][nt][2] * qscale, qv[kk][nt][3] * qscale);
        } else {
          qb[kk][nt][0] = pack_bf16x2(qv[kk][nt][0], qv[kk][nt][1]);
          qb[kk][nt][1] = pack_bf16x2(qv[kk][nt][2], qv[kk][nt][3]);
        }
      }
  }

  float o[KSTEPS][NT][4];
  float mrow[NT][2], lrow[NT][2];
#pragma unroll
  for (int mt = 0; mt < KSTEPS; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[mt][nt][e] = 0.f;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    mrow[nt][0] = mrow[nt][1] = -INFINITY;
    lrow[nt][0] = lrow[nt][1] = 0.f;
  }


  const int r0 = warp * 16;
  for (int it = 0; it < ntiles; ++it) {
    cp_async_wait<kStages - 2>();
    __syncthreads();
    {
      const int nxt = it + kStages - 1;
      if (nxt < ntiles) load_tile(nxt, nxt % kStages);
      cp_async_commit();
    }
    const int stage = it % kStages;
    const uint32_t ks = smem_u32(smem + stage * 2 * TILEB);
    const uint32_t vs = ks + TILEB;
    const int t0 = t_begin + it * kRows + r0;
    if (t0 >= t_end) continue;  // this warp's rows are past the end (uniform per warp)

    // ---- S^T = K . Q^T
    float s[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
    const int arow = r0 + (lane & 7) + ((lane >> 3) & 1) * 8;
    if (!FP8) {
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4(a0, a1, a2, a3, ks + arow * PITCH + (kk * 16 + (lane >> 4) * 8) * 2);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_bf16(s[nt], a0, a1, a2, a3, qb[kk][nt][0], qb[kk][nt][1]);
      }
    } else {
#pragma unroll
      for (int k2 = 0; k2 < KSTEPS / 2; ++k2) {
        uint32_t r0_, r1_, r2_, r3_;
        ldmatrix_x4(r0_, r1_, r2_, r3_, ks + arow * PITCH + k2 * 32 + (lane >> 4) * 16);
        const uint32_t x0 = e4m3x2_to_f16x2(r0_), x1 = e4m3x2_to_f16x2(r1_);
        const uint32_t x2 = e4m3x2_to_f16x2(r0_ >> 16), x3 = e4m3x2_to_f16x2(r1_ >> 16);
        const uint32_t y0 = e4m3x2_to_f16x2(r2_), y1 = e4m3x2_to_f16x2(r3_);
        const uint32_t y2 = e4m3x2_to_f16x2(r2_ >> 16), y3 = e4m3x2_to_f16x2(r3_ >> 16);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma_f16(s[nt], x0, x1, x2, x3, qb[2 * k2][nt][0], qb[2 * k2][nt][1]);
          mma_f16(s[nt], y0, y1, y2, y3, qb[2 * k2 + 1][nt][0], qb[2 * k2 + 1][nt][1]);
        }
      }
    }

    // ---- mask, online softmax (exp2 domain), P fragments
    const bool v0 = t0 + g < t_end, v1 = t0 + g + 8 < t_end;
    uint32_t pb[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      // mrow moves only when a score passes it (to that score + kHeadroomD); the head maxima
      // are reduced over the warp and the running sums rescaled only then
      float pv[4], a[2], c[2], mx[2];
      bool grow = false;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        a[j] = v0 ? s[nt][j] * score_mul : -INFINITY;
        c[j] = v1 ? s[nt][2 + j] * score_mul : -INFINITY;
        mx[j] = fmaxf(a[j], c[j]);
        grow |= mx[j] > mrow[nt][j];
      }
      if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], 4));
          mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], 8));
          mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], 16));
          const float mnew = mx[j] > mrow[nt][j] ? mx[j] + kHeadroomD : mrow[nt][j];
          const float alpha = mrow[nt][j] == -INFINITY ? 0.f : fast_exp2(mrow[nt][j] - mnew);
          mrow[nt][j] = mnew;
          lrow[nt][j] *= alpha;
#pragma unroll
          for (int mt = 0; mt < KSTEPS; ++mt) {
            o[mt][nt][j] *= alpha;
            o[mt][nt][2 + j] *= alpha;
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float muse = mrow[nt][j] == -INFINITY ? 0.f : mrow[nt][j];
        pv[j] = fast_exp2(a[j] - muse);
        pv[2 + j] = fast_exp2(c[j] - muse);
        lrow[nt][j] += pv[j] + pv[2 + j];
      }
      if (FP8) {
        pb[nt][0] = movmatrix_trans(pack_f16x2(pv[0], pv[1]));
        pb[nt][1] = movmatrix_trans(pack_f16x2(pv[2], pv[3]));
      } else {
        pb[nt][0] = movmatrix_trans(pack_bf16x2(pv[0], pv[1]));
        pb[nt][1] = movmatrix_trans(pack_bf16x2(pv[2], pv[3]));
      }
    }

    // ---- O^T += V^T . P^T
    if (!FP8) {
      const int vrow = r0 + (lane & 7) + (lane >> 4) * 8;
#pragma unroll
      for (int mt = 0; mt < KSTEPS; ++mt) {
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4_trans(a0, a1, a2, a3, vs + vrow * PITCH + (mt * 16 + ((lane >> 3) & 1) * 8) * 2);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_bf16(o[mt][nt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
      }
    } else {
      const int vrow = r0 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int m2 = 0; m2 < KSTEPS / 2; ++m2) {
        uint32_t r0_, r1_, r2_, r3_;
        ldmatrix_x4_trans(r0_, r1_, r2_, r3_, vs + vrow * PITCH + m2 * 32 + (lane >> 4) * 16);
        // r0: tokens 0-7, r1: tokens 8-15 of channel block [32*m2, +16); r2/r3: block +16.
        // Each holds (tok 2tq: ch 2g,2g+1 | tok 2tq+1: ch 2g,2g+1) as bytes 0..3.
        const uint32_t a0 = e4m3x2_to_f16x2(prmt(r0_, 0, 0x0020)), a1 = e4m3x2_to_f16x2(prmt(r0_, 0, 0x0031));
        const uint32_t a2 = e4m3x2_to_f16x2(prmt(r1_, 0, 0x0020)), a3 = e4m3x2_to_f16x2(prmt(r1_, 0, 0x0031));
        const uint32_t c0 = e4m3x2_to_f16x2(prmt(r2_, 0, 0x0020)), c1 = e4m3x2_to_f16x2(prmt(r2_, 0, 0x0031));
        const uint32_t c2 = e4m3x2_to_f16x2(prmt(r3_, 0, 0x0020)), c3 = e4m3x2_to_f16x2(prmt(r3_, 0, 0x0031));
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma_f16(o[2 * m2][nt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
          mma_f16(o[2 * m2 + 1][nt], c0, c1, c2, c3, pb[nt][0], pb[nt][1]);
        }
      }
    }
  }

  // ---- merge the warps: sum l over rows, then rescale to the CTA-wide max
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float l = lrow[nt][j];
      l += __shfl_xor_sync(0xffffffffu, l, 4);
      l += __shfl_xor_sync(0xffffffffu, l, 8);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      lrow[nt][j] = l;
    }
  cp_async_wait<0>();
  __syncthreads();
  float* red_m = reinterpret_cast<float*>(smem);   // [warps][NH]
  float* red_l = red_m + kWarps * NH;              // [warps][NH]
  float* red_o = red_l + kWarps * NH;              // [warps][NH][D]
  if (g == 0) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        red_m[warp * NH + nt * 8 + 2 * tq + j] = mrow[nt][j];
        red_l[warp * NH + nt * 8 + 2 * tq + j] = lrow[nt][j];
      }
  }
  __syncthreads();
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int h = nt * 8 + 2 * tq + j;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) M = fmaxf(M, red_m[w * NH + h]);
      const float f = (M == -INFINITY) ? 0.f : exp2f(mrow[nt][j] - M);
#pragma unroll
      for (int mt = 0; mt < KSTEPS; ++mt) {
        const int ca = FP8 ? mt * 16 + 2 * g : mt * 16 + g;
        const int cb = FP8 ? ca + 1 : ca + 8;
        red_o[(warp * NH + h) * D + ca] = o[mt][nt][j] * f;
        red_o[(warp * NH + h) * D + cb] = o[mt][nt][2 + j] * f;
      }
    }
  __syncthreads();
  if (p.merge) {
    // ---- merge with the slots of the pass this grid waits for. Phase A: TPH threads per
    // head turn the slot maxima into weights; phase B: thread = (head, 4 channels).
    griddep_wait();
    const int n = p.split_offset;
    constexpr int TPH = kWarps * 32 / NH;
    float* wts = red_o + kWarps * NH * D;  // [NH][n + 1]; slot n = this CTA
    float* sl = wts + NH * (n + 1);        // [NH] total sums
    // The group's rows are consecutive, so all their slots form one block of
    // nheads * split_stride * D floats: one bulk copy brings it into shared memory while
    // the weights are computed (when it fits; else the slots are read from global memory).
    const int64_t row0 = int64_t(b) * p.Hq + hk * p.G + h0;
    const uint32_t blk_off = (uint32_t((reinterpret_cast<uint8_t*>(sl + NH) - smem)) + 15u) & ~15u;
    const uint32_t blk_bytes = uint32_t(nheads) * uint32_t(p.split_stride) * uint32_t(D) * 4u;
    bool staged = blk_off + blk_bytes + 8u <= uint32_t(p.smem_bytes);
    const float* ob = reinterpret_cast<const float*>(smem + blk_off);
    const uint32_t mbar = smem_u32(smem + blk_off + blk_bytes);
    if (staged && threadIdx.x == 0) {
      mbar_init(mbar, 1);
      mbar_fence_init();
      mbar_arrive_expect_tx(mbar, blk_bytes);
      bulk_load(smem_u32(smem + blk_off), p.part_o + row0 * p.split_stride * D, blk_bytes, mbar);
    }
    {
      const int h = threadIdx.x / TPH, part = threadIdx.x % TPH;
      const int hq = hk * p.G + h0 + min(h, nheads - 1);
      const int64_t row = int64_t(b) * p.Hq + hq;
      const float* mr = p.part_m + row * p.split_stride;
      const float* lr = p.part_l + row * p.split_stride;
      float Mo = -INFINITY;  // this CTA's maximum (log2 units) and sum
#pragma unroll
      for (int w = 0; w < kWarps; ++w) Mo = fmaxf(Mo, red_m[w * NH + h]);
      float Lo = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) Lo += Mo == -INFINITY ? 0.f : red_l[w * NH + h] * exp2f(red_m[w * NH + h] - Mo);
      const float mo = Mo * kLn2;
      float Mx = mo;
      for (int s = part; s < n; s += TPH) Mx = fmaxf(Mx, __ldcg(mr + s));
#pragma unroll
      for (int d = 1; d < TPH; d <<= 1) Mx = fmaxf(Mx, __shfl_xor_sync(0xffffffffu, Mx, d));
      float L = 0.f;
      for (int s = part; s < n; s += TPH) {
        const float w = Mx == -INFINITY ? 0.f : __expf(__ldcg(mr + s) - Mx);
        wts[h * (n + 1) + s] = w;
        L = fmaf(__ldcg(lr + s), w, L);
      }
#pragma unroll
      for (int d = 1; d < TPH; d <<= 1) L += __shfl_xor_sync(0xffffffffu, L, d);
      if (part == 0) {
        const float wo = Mx == -INFINITY ? 0.f : __expf(mo - Mx);
        wts[h * (n + 1) + n] = wo;
        sl[h] = L + Lo * wo;
      }
    }
    // the staged slots never arrived: read them from global memory instead (the copy gets
    // one more bounded wait before the CTA exits, below)
    const bool lost = staged && !mbar_wait(mbar, 0);
    if (__syncthreads_or(lost)) {
      if (threadIdx.x == 0) atomicAdd(&g_merge_timeouts, 1u);
      staged = false;
    }
    constexpr int C4 = D / 4;
    for (int idx = threadIdx.x; idx < nheads * C4; idx += kWarps * 32) {
      const int h = idx / C4, c = 4 * (idx % C4);
      const int hq = hk * p.G + h0 + h;
      const int64_t row = int64_t(b) * p.Hq + hq;
      const float* wr = wts + h * (n + 1);
      float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float4 v = *reinterpret_cast<const float4*>(red_o + (w * NH + h) * D + c);
        O.x += v.x; O.y += v.y; O.z += v.z; O.w += v.w;
      }
      const float wo = wr[n];
      O.x *= wo; O.y *= wo; O.z *= wo; O.w *= wo;
      if (staged) {
        const float* orow = ob + int64_t(h) * p.split_stride * D + c;
#pragma unroll 6
        for (int s = 0; s < n; ++s) {
          const float4 v = *reinterpret_cast<const float4*>(orow + s * D);
          const float w = wr[s];
          O.x = fmaf(v.x, w, O.x); O.y = fmaf(v.y, w, O.y); O.z = fmaf(v.z, w, O.z); O.w = fmaf(v.w, w, O.w);
        }
      } else {
        const float* orow = p.part_o + row * p.split_stride * D + c;
#pragma unroll 6
        for (int s = 0; s < n; ++s) {
          const float4 v = __ldcg(reinterpret_cast<const float4*>(orow + int64_t(s) * D));
          const float w = wr[s];
          O.x = fmaf(v.x, w, O.x); O.y = fmaf(v.y, w, O.y); O.z = fmaf(v.z, w, O.z); O.w = fmaf(v.w, w, O.w);
        }
      }
      const float inv = 1.f / sl[h];
      const int64_t off = int64_t(b) * p.o_sb + int64_t(hq) * p.o_sh + c;
      store_out(p.out, p.out_dtype, off, O.x * inv);
      store_out(p.out, p.out_dtype, off + 1, O.y * inv);
      store_out(p.out, p.out_dtype, off + 2, O.z * inv);
      store_out(p.out, p.out_dtype, off + 3, O.w * inv);
    }
    if (lost) mbar_wait(mbar, 0);
    return;
  }
  for (int idx = threadIdx.x; idx < nheads * D; idx += kWarps * 32) {
    const int h = idx / D, c = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, red_m[w * NH + h]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = (M == -INFINITY) ? 0.f : exp2f(red_m[w * NH + h] - M);
      L += red_l[w * NH + h] * f;
      O += red_o[(w * NH + h) * D + c];
    }
    const int hq = hk * p.G + h0 + h;
    if (p.direct) {
      store_out(p.out, p.out_dtype, int64_t(b) * p.o_sb + int64_t(hq) * p.o_sh + c, O / L);
    } else {
      const int64_t pi = (int64_t(b) * p.Hq + hq) * p.split_stride + p.split_offset + split;
      p.part_o[pi * D + c] = O;
      if (c == 0) {
        p.part_m[pi] = M * kLn2;  // natural-log units of scaling*q.k
        p.part_l[pi] = L;
      }
    }
  }
  if (p.pdl) griddep_wait();
}

// Merge per-split partials. mode 0: final output O/L; mode 1: export (m, l, O) per (b,hq).
struct CombineParams {
  const float* m; const float* l; const float* o;  // [rows][n] and [rows][n][D]
  int rows, n, D, Hq;
  int64_t m_s0, o_s0;   // stride between the n partial sets (elements); contiguous rows inside
  void* out; int out_dtype; int64_t o_sb, o_sh;
  float* em; float* el; float* eo;  // export targets [rows], [rows], [rows][D]
  int mode;
  int ms_rows;          // 1: partials laid out [rows][n]; 0: [n][rows]
};

constexpr int kCombThreads = 256;

// One CTA per output row. Warp 0 turns the split maxima into weights; then thread
// (slice, c4) accumulates channels 4*c4..4*c4+3 over splits slice, slice+ns, ... with
// 16-byte loads (one warp reads a whole 512-byte partial row at D = 128), and the ns
// slice sums meet in shared memory. VEC4 needs D % 4 == 0 and 16-byte aligned partial
// rows; otherwise one channel per thread.
template <bool VEC4>
__global__ void __launch_bounds__(kCombThreads) lse_combine_kernel(const CombineParams p) {
  griddep_wait();  // partials of a programmatic predecessor (no-op after a plain launch)
  extern __shared__ __align__(16) float wsm[];  // [n4] weights, then [ns][D] slice sums
  const int row = blockIdx.x;
  __shared__ float sM, sL;
  auto midx = [&](int i) -> int64_t { return p.ms_rows ? int64_t(row) * p.n + i : int64_t(i) * p.m_s0 + row; };
  auto orow = [&](int i) -> int64_t {
    return p.ms_rows ? (int64_t(row) * p.n + i) * p.D : int64_t(i) * p.o_s0 + int64_t(row) * p.D;
  };
  if (threadIdx.x < 32) {
    float M = -INFINITY;
    for (int i = threadIdx.x; i < p.n; i += 32) M = fmaxf(M, p.m[midx(i)]);
    M = warp_max(M);
    float L = 0.f;
    for (int i = threadIdx.x; i < p.n; i += 32) {
      const float w = (M == -INFINITY) ? 0.f : __expf(p.m[midx(i)] - M);
      wsm[i] = w;
      L += p.l[midx(i)] * w;
    }
    L = warp_sum(L);
    if (threadIdx.x == 0) { sM = M; sL = L; }
  }
  __syncthreads();
  float* red = wsm + ((p.n + 3) & ~3);
  const int per = VEC4 ? p.D / 4 : p.D;  // threads per slice
  const int ns = kCombThreads / per;     // split slices (>= 1: D <= kCombThreads * (VEC4 ? 4 : 1))
  const int ci = threadIdx.x % per, sl = threadIdx.x / per;
  if (sl < ns) {
    if (VEC4) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
      for (int i = sl; i < p.n; i += ns) {
        const float4 v = *reinterpret_cast<const float4*>(p.o + orow(i) + 4 * ci);
        const float w = wsm[i];
        acc.x = fmaf(v.x, w, acc.x); acc.y = fmaf(v.y, w, acc.y);
        acc.z = fmaf(v.z, w, acc.z); acc.w = fmaf(v.w, w, acc.w);
      }
      reinterpret_cast<float4*>(red)[sl * per + ci] = acc;
    } else {
      float acc = 0.f;
#pragma unroll 4
      for (int i = sl; i < p.n; i += ns) acc = fmaf(p.o[orow(i) + ci], wsm[i], acc);
      red[sl * per + ci] = acc;
    }
  }
  __syncthreads();
  const int b = row / p.Hq, h = row % p.Hq;
  for (int c = threadIdx.x; c < p.D; c += kCombThreads) {
    float O = 0.f;
    for (int q = 0; q < ns; ++q) O += red[q * p.D + c];
    if (p.mode == 0) {
      store_out(p.out, p.out_dtype, int64_t(b) * p.o_sb + int64_t(h) * p.o_sh + c, O / sL);
    } else {
      p.eo[int64_t(row) * p.D + c] = O;
      if (c == 0) { p.em[row] = sM; p.el[row] = sL; }
    }
  }
}

// Launches the combine for c.rows rows (plain, or as a programmatic dependent).
int launch_combine_kernel(const CombineParams& c, cudaStream_t st, bool pdl) {
  if (c.rows == 0) return BD_OK;
  if (c.D <= 0 || c.D > kCombThreads * 4) return fail(BD_ERR_UNSUPPORTED, "combine supports head_dim up to 1024");
  const bool vec4 = c.D % 4 == 0 && (reinterpret_cast<uintptr_t>(c.o) & 15) == 0 && (c.ms_rows || c.o_s0 % 4 == 0) &&
                    c.D / 4 <= kCombThreads;
  const int per = vec4 ? c.D / 4 : c.D;
  if (per > kCombThreads) return fail(BD_ERR_UNSUPPORTED, "combine: head_dim not a multiple of 4 above 256");
  const int ns = kCombThreads / per;
  const size_t smem = (size_t((c.n + 3) & ~3) + size_t(ns) * c.D) * sizeof(float);
  auto kern = vec4 ? lse_combine_kernel<true> : lse_combine_kernel<false>;
  if (smem > 48 * 1024) {
    const int rc = cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
                              "cudaFuncSetAttribute(combine)");
    if (rc) return rc;
  }
  if (pdl) return launch_programmatic(kern, dim3(c.rows), dim3(kCombThreads), smem, st, c, "lse_combine_kernel launch");
  kern<<<c.rows, kCombThreads, smem, st>>>(c);
  return cuda_check(cudaGetLastError(), "lse_combine_kernel launch");
}

struct Plan {
  int D, NT, head_chunks, heads_per_chunk, n_splits, tiles_per_split;
  bool fp8;
};

int make_plan(const bd_tensor* q, const bd_tensor* k, Plan* pl, int target_ctas = 0) {
  const int64_t B = q->shape[0], Hq = q->shape[1], D = q->shape[2];
  const int64_t Hk = k->shape[1], S = k->shape[2];
  if (Hk <= 0 || Hq % Hk) return fail(BD_ERR_SHAPE, "H_q must be a multiple of H_k");
  if (D != 64 && D != 128) return fail(BD_ERR_UNSUPPORTED, "head_dim must be 64 or 128, got " + std::to_string(D));
  const int G = int(Hq / Hk);
  pl->D = int(D);
  pl->fp8 = k->dtype == BD_F8E4M3;
  pl->NT = G <= 8 ? 1 : 2;
  pl->heads_per_chunk = 8 * pl->NT;
  pl->head_chunks = (G + pl->heads_per_chunk - 1) / pl->heads_per_chunk;
  const int64_t ntiles = (S + kRows - 1) / kRows;
  const int64_t pairs = B * Hk * pl->head_chunks;
  const int64_t slots = target_ctas > 0 ? target_ctas : int64_t(dense_ctas_per_sm(pl->fp8)) * num_sms();
  int64_t splits = pairs >= slots ? 1 : slots / std::max<int64_t>(pairs, 1);
  splits = std::max<int64_t>(1, std::min<int64_t>(splits, std::max<int64_t>(ntiles, 1)));
  int64_t tps = ntiles > 0 ? (ntiles + splits - 1) / splits : 1;
  // at least 4 tiles (256 tokens) per split unless the caller fixed the CTA count: a short
  // context then keeps fewer, fuller splits, and the merge reads fewer partial rows
  if (target_ctas <= 0) tps = std::min<int64_t>(std::max<int64_t>(tps, 4), std::max<int64_t>(ntiles, 1));
  splits = ntiles > 0 ? (ntiles + tps - 1) / tps : 1;
  pl->n_splits = int(splits);
  pl->tiles_per_split = int(tps);
  return BD_OK;
}

size_t ws_bytes(const bd_tensor* q, const Plan& pl) {
  const size_t rows = size_t(q->shape[0]) * size_t(q->shape[1]);
  return rows * size_t(pl.n_splits) * (size_t(pl.D) + 2) * sizeof(float) + 256;
}

template <int D, int NT, bool FP8>
int launch_dense(const DenseParams& p, const Plan& pl, cudaStream_t st) {
  constexpr int ELT = FP8 ? 1 : 2;
  constexpr int PITCH = D * ELT + 16;
  size_t smem = size_t(kStages) * 2 * kRows * PITCH;
  size_t red = (2 * kWarps * 8 * NT + size_t(kWarps) * 8 * NT * D) * sizeof(float);
  if (p.merge) red += (size_t(8 * NT) * (p.split_offset + 1) + 8 * NT) * sizeof(float);
  smem = std::max(smem, red);
  DenseParams q = p;
  q.smem_bytes = int(smem);
  auto kern = dense_decode_kernel<D, NT, FP8>;
  static size_t attr_set[64] = {0};  // dynamic shared memory allowed so far, per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_set[dev & 63] < smem) {
    int rc = cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
                        "cudaFuncSetAttribute");
    if (rc) return rc;
    attr_set[dev & 63] = smem;
  }
  dim3 grid(pl.n_splits, p.Hk * pl.head_chunks, p.B);
  if (p.pdl) return launch_programmatic(kern, grid, dim3(kWarps * 32), smem, st, q, "dense_decode_kernel launch");
  kern<<<grid, kWarps * 32, smem, st>>>(q);
  return cuda_check(cudaGetLastError(), "dense_decode_kernel launch");
}

int dispatch_dense(const DenseParams& p, const Plan& pl, cudaStream_t st) {
  if (pl.D == 128) {
    if (pl.fp8) return pl.NT == 1 ? launch_dense<128, 1, true>(p, pl, st) : launch_dense<128, 2, true>(p, pl, st);
    return pl.NT == 1 ? launch_dense<128, 1, false>(p, pl, st) : launch_dense<128, 2, false>(p, pl, st);
  }
  if (pl.fp8) return pl.NT == 1 ? launch_dense<64, 1, true>(p, pl, st) : launch_dense<64, 2, true>(p, pl, st);
  return pl.NT == 1 ? launch_dense<64, 1, false>(p, pl, st) : launch_dense<64, 2, false>(p, pl, st);
}

int validate(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v) {
  int rc;
  if ((rc = check_tensor(q, "q", 3))) return rc;
  if ((rc = check_tensor(k, "k", 4))) return rc;
  if ((rc = check_tensor(v, "v", 4))) return rc;
  if (q->dtype != BD_BF16 && q->dtype != BD_F16 && q->dtype != BD_F32)
    return fail(BD_ERR_DTYPE, "q must be bf16, f16 or f32");
  if (k->dtype != v->dtype || (k->dtype != BD_BF16 && k->dtype != BD_F8E4M3))
    return fail(BD_ERR_DTYPE, "k and v must both be bf16 or both fp8 e4m3");
  if (k->dtype == BD_BF16 && q->dtype != BD_BF16)
    return fail(BD_ERR_DTYPE, "a bf16 KV cache needs a bf16 query");
  for (int i = 0; i < 4; ++i)
    if (k->shape[i] != v->shape[i]) return fail(BD_ERR_SHAPE, "k and v shapes differ");
  if (k->shape[0] != q->shape[0] || k->shape[3] != q->shape[2])
    return fail(BD_ERR_SHAPE, "q " + shape_str(q) + " does not match k " + shape_str(k));
  if (q->shape[2] > 1 && q->stride[2] != 1) return fail(BD_ERR_STRIDE, "q innermost dim must be contiguous");
  if ((rc = check_rows_aligned(k, "k"))) return rc;
  if ((rc = check_rows_aligned(v, "v"))) return rc;
  return BD_OK;
}

void fill_common(DenseParams& p, const bd_tensor* q, const bd_tensor* k, const bd_tensor* v, const Plan& pl,
                 float scaling) {
  p.q = q->data; p.q_sb = q->stride[0]; p.q_sh = q->stride[1]; p.q_dtype = q->dtype;
  p.k = static_cast<const uint8_t*>(k->data); p.k_sb = k->stride[0]; p.k_sh = k->stride[1]; p.k_ss = k->stride[2];
  p.v = static_cast<const uint8_t*>(v->data); p.v_sb = v->stride[0]; p.v_sh = v->stride[1]; p.v_ss = v->stride[2];
  p.B = int(q->shape[0]); p.Hq = int(q->shape[1]); p.Hk = int(k->shape[1]); p.G = p.Hq / p.Hk; p.S = int(k->shape[2]);
  p.head_chunks = pl.head_chunks; p.heads_per_chunk = pl.heads_per_chunk;
  p.tiles_per_split = pl.tiles_per_split; p.n_splits = pl.n_splits;
  p.split_offset = 0; p.split_stride = pl.n_splits;
  p.scale_log2 = scaling * kLog2e;
}

}  // namespace

int dense_split_count(int64_t B, int64_t Hq, int64_t Hk, int64_t S, int64_t D, int target_ctas) {
  bd_tensor q{}, k{};
  q.ndim = 3; q.shape[0] = B; q.shape[1] = Hq; q.shape[2] = D;
  k.ndim = 4; k.shape[0] = B; k.shape[1] = Hk; k.shape[2] = S; k.shape[3] = D; k.dtype = BD_BF16;
  Plan pl;
  if (make_plan(&q, &k, &pl, target_ctas)) return -1;
  return pl.n_splits;
}

int launch_dense_partials(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v, float scaling,
                          const Partials& part, int split_offset, int nsplit_here, cudaStream_t st, bool pdl) {
  int rc;
  if ((rc = validate(q, k, v))) return rc;
  Plan pl;
  if ((rc = make_plan(q, k, &pl))) return rc;
  // force the caller's split count
  const int64_t S = k->shape[2];
  const int64_t ntiles = (S + kRows - 1) / kRows;
  const int64_t tps = ntiles > 0 ? (ntiles + nsplit_here - 1) / nsplit_here : 1;
  pl.tiles_per_split = int(tps);
  pl.n_splits = nsplit_here;
  DenseParams p{};
  fill_common(p, q, k, v, pl, scaling);
  p.part_m = part.m; p.part_l = part.l; p.part_o = part.o;
  p.split_offset = split_offset; p.split_stride = part.nsplit;
  p.direct = 0;
  p.pdl = pdl ? 1 : 0;
  return dispatch_dense(p, pl, st);
}

int launch_dense_merge(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v, float scaling,
                       const Partials& part, int split_offset, const bd_tensor* out, cudaStream_t st) {
  int rc;
  if ((rc = validate(q, k, v))) return rc;
  Plan pl;
  if ((rc = make_plan(q, k, &pl))) return rc;
  if (pl.D % 4) return fail(BD_ERR_UNSUPPORTED, "merge needs head_dim % 4 == 0");
  const int64_t S = k->shape[2];
  pl.tiles_per_split = int(std::max<int64_t>(1, (S + kRows - 1) / kRows));
  pl.n_splits = 1;
  DenseParams p{};
  fill_common(p, q, k, v, pl, scaling);
  p.part_m = part.m; p.part_l = part.l; p.part_o = part.o;
  p.split_offset = split_offset; p.split_stride = part.nsplit;
  p.out = out->data; p.out_dtype = out->dtype; p.o_sb = out->stride[0]; p.o_sh = out->stride[1];
  p.direct = 0;
  p.pdl = 1;
  p.merge = 1;
  return dispatch_dense(p, pl, st);
}

int launch_combine_export(const Partials& part, int B, int Hq, int D, float* em, float* el, float* eo,
                          cudaStream_t st, bool pdl) {
  CombineParams c{};
  c.m = part.m; c.l = part.l; c.o = part.o;
  c.rows = B * Hq; c.n = part.nsplit; c.D = D; c.Hq = Hq; c.ms_rows = 1;
  c.mode = 1;
  c.em = em; c.el = el; c.eo = eo;
  return launch_combine_kernel(c, st, pdl);
}

int launch_combine(const Partials& part, int B, int Hq, int D, const bd_tensor* out, cudaStream_t st, bool pdl) {
  CombineParams c{};
  c.m = part.m; c.l = part.l; c.o = part.o;
  c.rows = B * Hq; c.n = part.nsplit; c.D = D; c.Hq = Hq; c.ms_rows = 1;
  c.out = out->data; c.out_dtype = out->dtype; c.o_sb = out->stride[0]; c.o_sh = out->stride[1];
  c.mode = 0;
  return launch_combine_kernel(c, st, pdl);
}

// ---- static scratch for bd_decode_attn_noalloc --------------------------------------
// Some callers have no way to allocate device memory for us: a serving runtime that
// reserves all of HBM for its KV pages at start-up and forbids later cudaMalloc, or a
// plain C / FFI host that only owns the q/k/v/out buffers. For them the split partials
// live in this fixed array, which every GPU that loads the library keeps (4 MiB) until
// the process exits. In host code the symbol is only a stand-in, so its device address
// is looked up with cudaGetSymbolAddress on the calling device.
//
// Size: a plan that splits at all targets two CTAs per SM (three for fp8 caches), so it
// holds at most 3 x SMs CTAs x 16 heads of (D + 2) floats, D <= 128, plus 256 bytes of
// alignment slack: 24,960 bytes per SM. 4 MiB therefore covers every plan on parts with up
// to 168 SMs (B200: 148); a larger plan is rejected with BD_ERR_UNSUPPORTED before any launch.
constexpr size_t kStaticScratchBytes = size_t(4) << 20;
static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];
static std::mutex g_scratch_mu;
static void* g_scratch_addr[64] = {nullptr};

// The address is looked up again on every call made outside a stream capture, so a
// device reset (which reloads the module at a new address) never leaves a stale pointer;
// a call made while `st` is capturing uses the address of the device's last uncaptured call.
int static_scratch_address(cudaStream_t st, void** ptr) {
  int dev = 0;
  int rc = cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= 64) return fail(BD_ERR_UNSUPPORTED, "device index out of range for the static scratch");
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if ((rc = cuda_check(cudaStreamIsCapturing(st, &cap), "cudaStreamIsCapturing"))) return rc;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (cap == cudaStreamCaptureStatusNone) {
    void* a = nullptr;
    if ((rc = cuda_check(cudaGetSymbolAddress(&a, g_decode_scratch), "cudaGetSymbolAddress(static scratch)")))
      return rc;
    g_scratch_addr[dev] = a;
  } else if (!g_scratch_addr[dev]) {
    return fail(BD_ERR_VALUE, "bd_decode_attn_noalloc: make one call on this device outside stream capture first");
  }
  *ptr = g_scratch_addr[dev];
  return BD_OK;
}

}  // namespace bd

namespace bd {
// host read of this file's wait-timeout counter (-1 on failure)
long long merge_wait_timeouts() {
  unsigned int v = 0;
  return cudaMemcpyFromSymbol(&v, g_merge_timeouts, sizeof v) == cudaSuccess ? (long long)v : -1;
}
}  // namespace bd

extern "C" {

size_t bd_decode_attn_workspace(const bd_tensor* q, const bd_tensor* k) {
  if (bd::check_tensor(q, "q", 3) || bd::check_tensor(k, "k", 4)) return 0;
  bd::Plan pl;
  if (bd::make_plan(q, k, &pl)) return 0;
  return bd::ws_bytes(q, pl);
}

int bd_decode_attn(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v, const bd_tensor* out, float scaling,
                   void* workspace, size_t workspace_bytes, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if ((rc = validate(q, k, v))) return rc;
  if ((rc = check_tensor(out, "out", 3))) return rc;
  if (out->dtype != BD_BF16 && out->dtype != BD_F16 && out->dtype != BD_F32)
    return fail(BD_ERR_DTYPE, "out must be bf16, f16 or f32");
  for (int i = 0; i < 3; ++i)
    if (out->shape[i] != q->shape[i]) return fail(BD_ERR_SHAPE, "out shape must equal q shape");
  if (out->stride[2] != 1) return fail(BD_ERR_STRIDE, "out innermost dim must be contiguous");
  Plan pl;
  if ((rc = make_plan(q, k, &pl))) return rc;
  if (q->shape[0] == 0 || q->shape[1] == 0) return BD_OK;
  DenseParams p{};
  fill_common(p, q, k, v, pl, scaling);
  p.out = out->data; p.out_dtype = out->dtype; p.o_sb = out->stride[0]; p.o_sh = out->stride[1];
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (pl.n_splits == 1) {
    p.direct = 1;
    return dispatch_dense(p, pl, st);
  }
  const size_t need = ws_bytes(q, pl);
  if (!workspace || workspace_bytes < need)
    return fail(BD_ERR_WORKSPACE, "need " + std::to_string(need) + " workspace bytes");
  const size_t rows = size_t(p.B) * p.Hq;
  float* base = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  p.part_m = base;
  p.part_l = base + rows * pl.n_splits;
  p.part_o = base + 2 * rows * pl.n_splits;
  p.direct = 0;
  if ((rc = dispatch_dense(p, pl, st))) return rc;
  CombineParams c{};
  c.m = p.part_m; c.l = p.part_l; c.o = p.part_o;
  c.rows = int(rows); c.n = pl.n_splits; c.D = pl.D; c.Hq = p.Hq; c.ms_rows = 1;
  c.out = out->data; c.out_dtype = out->dtype; c.o_sb = out->stride[0]; c.o_sh = out->stride[1];
  c.mode = 0;
  return launch_combine_kernel(c, st, true);
}

// Variant of bd_decode_attn for callers that cannot hand us a workspace: its split
// partials go to a fixed, file-scope device buffer instead (see static_scratch_address).
int bd_decode_attn_noalloc(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v, const bd_tensor* out,
                           float scaling, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if ((rc = validate(q, k, v))) return rc;
  Plan pl;
  if ((rc = make_plan(q, k, &pl))) return rc;
  if (pl.n_splits == 1 || q->shape[0] * q->shape[1] == 0)
    return bd_decode_attn(q, k, v, out, scaling, nullptr, 0, stream);  // no scratch needed
  const size_t need = ws_bytes(q, pl);
  if (need > kStaticScratchBytes)
    return fail(BD_ERR_UNSUPPORTED, "this call needs " + std::to_string(need) +
                                        " bytes of split scratch but the static scratch holds " +
                                        std::to_string(kStaticScratchBytes) +
                                        "; use bd_decode_attn with a caller workspace");
  void* scratch = nullptr;
  if ((rc = static_scratch_address(reinterpret_cast<cudaStream_t>(stream), &scratch))) return rc;
  return bd_decode_attn(q, k, v, out, scaling, scratch, kStaticScratchBytes, stream);
}

int bd_decode_attn_partial(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v, float scaling,
                           const bd_tensor* m, const bd_tensor* l, const bd_tensor* o, void* workspace,
                           size_t workspace_bytes, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if ((rc = validate(q, k, v))) return rc;
  if ((rc = check_tensor(m, "m", 2, BD_F32)) || (rc = check_tensor(l, "l", 2, BD_F32)) ||
      (rc = check_tensor(o, "o", 3, BD_F32)))
    return rc;
  const int64_t B = q->shape[0], Hq = q->shape[1], D = q->shape[2];
  if (m->shape[0] != B || m->shape[1] != Hq || l->shape[0] != B || l->shape[1] != Hq || o->shape[0] != B ||
      o->shape[1] != Hq || o->shape[2] != D)
    return fail(BD_ERR_SHAPE, "m,l must be [B,Hq] and o [B,Hq,D]");
  if (m->stride[1] != 1 || m->stride[0] != Hq || l->stride[1] != 1 || l->stride[0] != Hq || o->stride[2] != 1 ||
      o->stride[1] != D || o->stride[0] != Hq * D)
    return fail(BD_ERR_STRIDE, "m, l, o must be contiguous");
  Plan pl;
  if ((rc = make_plan(q, k, &pl))) return rc;
  if (B == 0 || Hq == 0) return BD_OK;
  const size_t need = ws_bytes(q, pl);
  if (!workspace || workspace_bytes < need)
    return fail(BD_ERR_WORKSPACE, "need " + std::to_string(need) + " workspace bytes");
  DenseParams p{};
  fill_common(p, q, k, v, pl, scaling);
  const size_t rows = size_t(B) * Hq;
  float* base = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  p.part_m = base;
  p.part_l = base + rows * pl.n_splits;
  p.part_o = base + 2 * rows * pl.n_splits;
  p.direct = 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if ((rc = dispatch_dense(p, pl, st))) return rc;
  CombineParams c{};
  c.m = p.part_m; c.l = p.part_l; c.o = p.part_o;
  c.rows = int(rows); c.n = pl.n_splits; c.D = int(D); c.Hq = int(Hq); c.ms_rows = 1;
  c.mode = 1;
  c.em = static_cast<float*>(m->data); c.el = static_cast<float*>(l->data); c.eo = static_cast<float*>(o->data);
  return launch_combine_kernel(c, st, true);
}

int bd_lse_combine(const bd_tensor* m, const bd_tensor* l, const bd_tensor* o, const bd_tensor* out,
                   bd_stream_t stream) {
  using namespace bd;
  int rc;
  if ((rc = check_tensor(m, "m", 3, BD_F32)) || (rc = check_tensor(l, "l", 3, BD_F32)) ||
      (rc = check_tensor(o, "o", 4, BD_F32)) || (rc = check_tensor(out, "out", 3)))
    return rc;
  const int64_t n = m->shape[0], B = m->shape[1], Hq = m->shape[2], D = o->shape[3];
  if (l->shape[0] != n || l->shape[1] != B || l->shape[2] != Hq || o->shape[0] != n || o->shape[1] != B ||
      o->shape[2] != Hq || out->shape[0] != B || out->shape[1] != Hq || out->shape[2] != D)
    return fail(BD_ERR_SHAPE, "shapes must be m,l [n,B,Hq], o [n,B,Hq,D], out [B,Hq,D]");
  if (m->stride[2] != 1 || m->stride[1] != Hq || l->stride[2] != 1 || l->stride[1] != Hq ||
      m->stride[0] != l->stride[0] || o->stride[3] != 1 || o->stride[2] != D || o->stride[1] != Hq * D ||
      out->stride[2] != 1)
    return fail(BD_ERR_STRIDE, "m, l, o must be contiguous within each shard");
  if (out->dtype != BD_BF16 && out->dtype != BD_F16 && out->dtype != BD_F32)
    return fail(BD_ERR_DTYPE, "out must be bf16, f16 or f32");
  if (n <= 0 || n > 4096) return fail(BD_ERR_VALUE, "shard count must be in [1, 4096]");
  if (B * Hq == 0) return BD_OK;
  CombineParams c{};
  c.m = static_cast<const float*>(m->data); c.l = static_cast<const float*>(l->data);
  c.o = static_cast<const float*>(o->data);
  c.rows = int(B * Hq); c.n = int(n); c.D = int(D); c.Hq = int(Hq);
  c.m_s0 = m->stride[0]; c.o_s0 = o->stride[0]; c.ms_rows = 0;
  c.out = out->data; c.out_dtype = out->dtype; c.o_sb = out->stride[0]; c.o_sh = out->stride[1];
  c.mode = 0;
  return launch_combine_kernel(c, reinterpret_cast<cudaStream_t>(stream), false);
}

}  // extern "C"
