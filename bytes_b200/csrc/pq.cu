// PQ-LUT decode attention family, LUT build and PQ encode.
//
// References (saifmb0/bytes, src/attention_kernels.py):
//   decode_attn_pq_lut      :301-392  scores = sum_j LUT[b,hq,j,code_j] (scale folded in LUT)
//   decode_attn_pq_lut_kv   :397-500  + PQ-reconstructed values
//   paged_attn_pq_lut_kv    :505-619  + block table / context lengths
//   decode_attn_pq_lut_asym :625-750  + exact outlier channels q_out.k_out, fp8/bf16 V
//   paged_attn_pq_lut_asym  :756-898
//   sparse_score_pq_lut_asym:909-984  scores only
//   decode_attn_dequant     :187-296  (served as LUT = q_split . centroids, then the LUT path)
// and ProductQuantizer.quantize (src/quantization.py:160-211), the LUT einsum of
// benchmarks/test_correctness.py:181-182. Config-2 extension: int8 V with a per-token
// f16 scale.
//
// Decode design (one CTA = (batch, KV head, chunk of 4 query heads, token split), 8 warps):
//  * The chunk's LUT sits in shared memory as [M][K][4 heads] fp32, so one 8-byte load
//    returns a head pair; codes (and outlier keys, values) stream in 128-token tiles
//    through a cp.async pipeline, 16 tokens per warp.
//  * Lane (g, tq) scores tokens g and g+8 for head pair tq&1 over half of the subspaces
//    and combines halves by shuffle, which leaves the scores exactly in the
//    accumulator-fragment layout of the dense kernel: online softmax, a movmatrix
//    transpose of P, then O^T += V^T . P^T on the tensor cores (mma.sync).
//  * V as bf16 (ldmatrix.trans), fp8 / int8 (ldmatrix.trans on byte pairs, widened to f16
//    exactly: e4m3 by cvt, int8 by the 0x6400|(x^0x80) = 1152+x bit pattern minus 1152),
//    or PQ-reconstructed into an f16 tile.
#include "common.cuh"
#include "decode_shared.cuh"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace bd {
namespace {

constexpr int kPW = 8;              // warps per CTA
constexpr int kPRows = 16 * kPW;    // tokens per tile
constexpr int kPStages = 2;  // 2 stages: the LUT chunk plus two tiles fit twice per SM
constexpr int kHC = 4;              // query heads per CTA
constexpr float kLog2eP = 1.4426950408889634f;
constexpr float kLn2P = 0.6931471805599453f;
constexpr float kPHeadroom = 4.f;  // log2 headroom of the lazily moved softmax reference

enum VKind { V_BF16 = 0, V_FP8 = 1, V_INT8 = 2, V_PQ = 3, V_NONE = 4, V_F16 = 5 };

struct PqParams {
  const float* lut; int64_t l_sb, l_sh, l_sm, l_sk;
  const uint8_t* codes; int64_t c_sb, c_sh, c_ss, c_sm;
  const uint16_t* kout; int64_t ko_sb, ko_sh, ko_ss, ko_sc; int ko_dtype;  // bf16 / f16
  const void* qout; int64_t qo_sb, qo_sh, qo_sc; int qo_dtype;
  int C;  // outlier channels (<= 8)
  const uint8_t* v; int64_t v_sb, v_sh, v_ss;                     // elements
  const __half* vsc; int64_t vs_sb, vs_sh, vs_ss;                 // int8 per-token scale
  const uint8_t* vidx; int64_t vi_sb, vi_sh, vi_ss, vi_sm;        // PQ value codes
  const float* vcent; int64_t vc_sm, vc_sk, vc_sd; int Mv, Kv, dsv;
  const int32_t* btab; int64_t bt_sb, bt_ss; const int32_t* clens; int bsz;
  int B, Hq, Hk, G, S, M, K, D;
  int head_chunks, ntiles, n_splits;  // split s owns tiles [s*ntiles/n_splits, (s+1)*ntiles/n_splits)
  float* scores_out; int64_t so_sb, so_sh;  // V_NONE mode
  // M = 16, K = 256: the LUT re-laid out per (batch, KV head, head chunk) as [K][M][4 heads]
  // (pq_lut_regroup_kernel), so one 16-byte read returns the four heads of a lookup
  const float4* lut_t;
  float* part_m; float* part_l; float* part_o;
};

struct PqSmem {
  int lut_bytes, codes_pitch, codes_bytes, kout_pitch, kout_bytes, v_pitch, v_bytes, vs_bytes, stage, recon_bytes;
  int off_stages;                          // first stage, past the LUT
  int off_codes, off_kout, off_v, off_vs;  // regions inside a stage
};

__host__ __device__ inline int round16(int x) { return (x + 15) & ~15; }

// tma: the tensor-map form (1-byte values, D = 128, no outliers, not paged): values first
// in 128-byte rows under the 128-byte swizzle, then codes, then value scales; stages start
// on 1024-byte boundaries.
__host__ __device__ inline PqSmem pq_smem(int vk, int M, int K, int C, int D, int Mv, bool tma = false) {
  PqSmem s{};
  s.lut_bytes = M * K * kHC * 4;
  s.codes_pitch = round16(M);
  s.codes_bytes = kPRows * s.codes_pitch;
  s.kout_pitch = C > 0 ? 16 : 0;  // up to 8 x 2-byte outlier channels per token
  s.kout_bytes = kPRows * s.kout_pitch;
  int vrow = 0;
  if (vk == V_BF16 || vk == V_F16) vrow = D * 2;
  else if (vk == V_FP8 || vk == V_INT8) vrow = D;
  else if (vk == V_PQ) vrow = round16(Mv);
  s.v_pitch = vk == V_PQ ? vrow : (vrow ? vrow + 16 : 0);
  s.v_bytes = kPRows * s.v_pitch;
  s.vs_bytes = vk == V_INT8 ? kPRows * 2 : 0;
  s.recon_bytes = vk == V_PQ ? kPRows * (D * 2 + 16) : 0;
  if (tma) {
    s.v_pitch = D;
    s.v_bytes = kPRows * D;
    s.off_v = 0;
    s.off_codes = s.v_bytes;
    s.off_kout = s.off_codes + s.codes_bytes;
    s.off_vs = s.off_kout + s.kout_bytes;
    s.stage = (s.off_vs + s.vs_bytes + 1023) & ~1023;
    s.off_stages = (s.lut_bytes + 1023) & ~1023;
  } else {
    s.off_codes = 0;
    s.off_kout = s.codes_bytes;
    s.off_v = s.off_kout + s.kout_bytes;
    s.off_vs = s.off_v + s.v_bytes;
    s.stage = s.off_vs + s.vs_bytes;
    s.off_stages = s.lut_bytes;
  }
  return s;
}

// TMA waits that ran past their iteration limit (a non-zero count means a result is wrong)
__device__ unsigned int g_pq_tma_timeouts = 0;

// (a.x + b.x, a.y + b.y), both rounded to nearest: one paired fp32 add
__device__ __forceinline__ float2 add_f32x2(float2 a, float2 b) {
  unsigned long long x, y, z;
  x = (static_cast<unsigned long long>(__float_as_uint(a.y)) << 32) | __float_as_uint(a.x);
  y = (static_cast<unsigned long long>(__float_as_uint(b.y)) << 32) | __float_as_uint(b.x);
  asm("add.rn.f32x2 %0, %1, %2;\n" : "=l"(z) : "l"(x), "l"(y));
  return make_float2(__uint_as_float(uint32_t(z)), __uint_as_float(uint32_t(z >> 32)));
}

__device__ __forceinline__ float ld16f(const uint16_t* p, int64_t off, int dt) {
  const uint16_t u = p[off];
  return dt == BD_BF16 ? __uint_as_float(uint32_t(u) << 16) : __half2float(__ushort_as_half(u));
}

template <int VK, bool PAGED, bool OUTL, int D, bool TMA>
__global__ void __launch_bounds__(kPW * 32, 2)
    pq_decode_kernel(const PqParams p, const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ CUtensorMap tm_codes, const __grid_constant__ CUtensorMap tm_vs) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // TMA stages sit on the swizzle atom: align the working base by hand (the launch adds 1 KB)
  uint8_t* smem = TMA ? smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u) : smem_raw;
  griddep_launch_dependents();  // the combine queued behind may start launching (it waits for this grid)
  constexpr int KSTEPS = D / 16;
  const PqSmem L = pq_smem(VK, p.M, p.K, OUTL ? p.C : 0, D, p.Mv, TMA);
  float* lut_s = reinterpret_cast<float*>(smem);
  uint8_t* stages = smem + L.off_stages;
  uint8_t* recon = stages + kPStages * L.stage;
  const uint32_t bar0 = smem_u32(stages + kPStages * L.stage);  // TMA: one mbarrier per stage
  if (TMA) {
    if (threadIdx.x == 0) {
      for (int s = 0; s < kPStages; ++s) mbar_init(bar0 + 8 * s, 1);
      mbar_fence_init();
    }
    __syncthreads();
  }

  const int split = blockIdx.x;
  const int hk = blockIdx.y / p.head_chunks;
  const int chunk = blockIdx.y % p.head_chunks;
  const int b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int h0 = chunk * kHC;
  const int nheads = min(kHC, p.G - h0);
  const int S_b = PAGED ? min(p.S, p.clens[b]) : p.S;
  const int tile0 = int(int64_t(split) * p.ntiles / p.n_splits);
  const int t_begin = tile0 * kPRows;
  const int t_end = min(S_b, int(int64_t(split + 1) * p.ntiles / p.n_splits) * kPRows);
  const int ntiles = t_end > t_begin ? (t_end - t_begin + kPRows - 1) / kPRows : 0;

  // ---- LUT of the chunk's heads -> smem: the regrouped [K][M][4] copy when there is one
  // (one contiguous 64 KB block, copied after the first tiles are in flight, below), else
  // [M][K][4] from the caller's layout; rows of a head are read four entries at a time when
  // they are contiguous and 16-byte aligned
  if (!p.lut_t) {
    const int MK = p.M * p.K;
    const bool vec = p.l_sk == 1 && p.l_sm == p.K && (p.K & 3) == 0 && (p.l_sh & 3) == 0 && (p.l_sb & 3) == 0 &&
                     (reinterpret_cast<uintptr_t>(p.lut) & 15) == 0;
    for (int h = 0; h < kHC; ++h) {
      const float* src = p.lut + int64_t(b) * p.l_sb + int64_t(hk * p.G + h0 + min(h, nheads - 1)) * p.l_sh;
      if (vec) {
        for (int i = threadIdx.x; i < MK / 4; i += kPW * 32) {
          const float4 x = h < nheads ? reinterpret_cast<const float4*>(src)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
          float* d = lut_s + (4 * i) * kHC + h;
          d[0] = x.x; d[kHC] = x.y; d[2 * kHC] = x.z; d[3 * kHC] = x.w;
        }
      } else {
        for (int i = threadIdx.x; i < MK; i += kPW * 32) {
          const int c = i % p.K, j = i / p.K;
          lut_s[i * kHC + h] = h < nheads ? src[int64_t(j) * p.l_sm + int64_t(c) * p.l_sk] : 0.f;
        }
      }
    }
  }
  // outlier query of the lane's head pair (tq & 1): heads 2hp, 2hp+1
  const int hp = tq & 1;
  float qo[2][8];
  if (OUTL) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int h = 2 * hp + e;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float x = 0.f;
        if (h < nheads && c < p.C) {
          const int64_t off = int64_t(b) * p.qo_sb + int64_t(hk * p.G + h0 + h) * p.qo_sh + int64_t(c) * p.qo_sc;
          if (p.qo_dtype == BD_BF16) x = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.qout)[off]);
          else if (p.qo_dtype == BD_F16) x = __half2float(reinterpret_cast<const __half*>(p.qout)[off]);
          else x = reinterpret_cast<const float*>(p.qout)[off];
        }
        qo[e][c] = x;
      }
    }
  }

  // token -> (base row offset) for codes/outliers/values, paged or not
  auto row_of = [&](int t, int64_t sb, int64_t sh, int64_t ss) -> int64_t {
    if (PAGED) {
      const int blk = p.btab[int64_t(b) * p.bt_sb + int64_t(t / p.bsz) * p.bt_ss];
      return int64_t(blk) * sb + int64_t(hk) * sh + int64_t(t % p.bsz) * ss;
    }
    return int64_t(b) * sb + int64_t(hk) * sh + int64_t(t) * ss;
  };

  auto load_tile = [&](int tile, int stage) {
    const int t0 = t_begin + tile * kPRows;
    uint8_t* st = stages + stage * L.stage;
    const uint32_t sb = smem_u32(st);
    if (TMA) {
      // one thread moves the tile; rows past the sequence arrive as zeros and rows past the
      // split are masked by the token bounds below
      if (threadIdx.x == 0) {
        const uint32_t bar = bar0 + 8 * stage;
        mbar_arrive_expect_tx(bar, uint32_t(L.v_bytes + L.codes_bytes + L.vs_bytes));
        tma_load_4d(sb + L.off_v, &tm_v, 0, t0, hk, b, bar);
        tma_load_4d(sb + L.off_codes, &tm_codes, 0, t0, hk, b, bar);
        if (VK == V_INT8) tma_load_3d(sb + L.off_vs, &tm_vs, t0, hk, b, bar);
      }
      return;
    }
    // codes: M bytes per token (M <= 16 -> one 16-byte chunk; else several)
    const int cch = L.codes_pitch / 16;
    for (int c = threadIdx.x; c < kPRows * cch; c += kPW * 32) {
      const int r = c / cch, cc = c % cch;
      const int t = t0 + r;
      const bool ok = t < t_end;
      const int nbytes = ok ? max(0, min(16, p.M - cc * 16)) : 0;
      const uint8_t* src = p.codes + (ok ? row_of(t, p.c_sb, p.c_sh, p.c_ss) : 0) + cc * 16;
      // byte-granular copy of possibly unaligned rows
      if (nbytes == 16 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        cp_async16(sb + L.off_codes + r * L.codes_pitch + cc * 16, src, 16);
      } else {
        for (int e = 0; e < 16; ++e) st[L.off_codes + r * L.codes_pitch + cc * 16 + e] = e < nbytes ? src[e] : 0;
      }
    }
    if (OUTL) {
      for (int r = threadIdx.x; r < kPRows; r += kPW * 32) {
        const int t = t0 + r;
        uint16_t* dst = reinterpret_cast<uint16_t*>(st + L.off_kout + r * L.kout_pitch);
        if (t < t_end) {
          const uint16_t* src = p.kout + row_of(t, p.ko_sb, p.ko_sh, p.ko_ss);
          for (int c = 0; c < 8; ++c) dst[c] = c < p.C ? src[int64_t(c) * p.ko_sc] : 0;
        } else {
          for (int c = 0; c < 8; ++c) dst[c] = 0;
        }
      }
    }
    uint8_t* vst = st + L.off_v;
    if (VK == V_BF16 || VK == V_F16 || VK == V_FP8 || VK == V_INT8) {
      constexpr int ELT = (VK == V_BF16 || VK == V_F16) ? 2 : 1;
      constexpr int CH = D * ELT / 16;
      for (int c = threadIdx.x; c < kPRows * CH; c += kPW * 32) {
        const int r = c / CH, cc = c % CH;
        const int t = t0 + r;
        const bool ok = t < t_end;
        const uint8_t* src = p.v + (ok ? row_of(t, p.v_sb, p.v_sh, p.v_ss) : 0) * ELT + cc * 16;
        cp_async16(sb + L.off_v + r * L.v_pitch + cc * 16, src, ok ? 16 : 0);
      }
      if (VK == V_INT8) {
        __half* vs = reinterpret_cast<__half*>(st + L.off_vs);
        for (int r = threadIdx.x; r < kPRows; r += kPW * 32) {
          const int t = t0 + r;
          vs[r] = t < t_end ? p.vsc[int64_t(b) * p.vs_sb + int64_t(hk) * p.vs_sh + int64_t(t) * p.vs_ss]
                            : __float2half(0.f);
        }
      }
    } else if (VK == V_PQ) {
      for (int i = threadIdx.x; i < kPRows * L.v_pitch; i += kPW * 32) {
        const int r = i / L.v_pitch, j = i % L.v_pitch;
        const int t = t0 + r;
        vst[i] = (t < t_end && j < p.Mv) ? p.vidx[row_of(t, p.vi_sb, p.vi_sh, p.vi_ss) + int64_t(j) * p.vi_sm] : 0;
      }
    }
  };

  float o[KSTEPS][4];
  // int8 values enter the MMA as 1152 + x (the f16 halves 0x64XX, XX = x ^ 0x80); oc
  // accumulates 1152 * sum_t P'_t with the same f16 P' (one MMA of a constant operand per
  // tile) and is subtracted from every channel at the end
  float oc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int mt = 0; mt < KSTEPS; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};

#pragma unroll
  for (int s = 0; s < kPStages - 1; ++s) {
    if (s < ntiles) load_tile(s, s);
    cp_async_commit();
  }
  if (p.lut_t) {
    // the regrouped LUT is written by the kernel this grid is a programmatic dependent of:
    // the first tiles above are already in flight while it finishes
    griddep_wait();
    const float4* src = p.lut_t + ((int64_t(b) * p.Hk + hk) * p.head_chunks + chunk) * (256 * 16);
    for (int i = threadIdx.x; i < 256 * 16; i += kPW * 32) cp_async16(smem_u32(lut_s) + i * 16, src + i, 16);
    cp_async_commit();
    cp_async_wait<0>();
  }
  __syncthreads();  // LUT visible

  const int jmid = (p.M + 1) / 2;
  const int jlo = (tq >> 1) ? jmid : 0, jhi = (tq >> 1) ? p.M : jmid;
  const int r0 = warp * 16;
  for (int it = 0; it < ntiles; ++it) {
    bool lost = false;
    if (TMA) lost = !mbar_wait(bar0 + 8 * (it % kPStages), (it / kPStages) & 1);
    else cp_async_wait<kPStages - 2>();
    if (__syncthreads_or(lost)) {
      // a tile copy never completed: one more bounded wait for every tile copy still in
      // flight (none may land in shared memory after this CTA exits), then mark this CTA's
      // partials as failed (NaN: the merged output is NaN) and count the event
      if (threadIdx.x == 0) atomicAdd(&g_pq_tma_timeouts, 1u);
      for (int t = it; t < min(ntiles, it + kPStages - 1); ++t) mbar_wait(bar0 + 8 * (t % kPStages), (t / kPStages) & 1);
      if (VK != V_NONE) {
        for (int idx = threadIdx.x; idx < nheads * D; idx += kPW * 32) {
          const int64_t pi = (int64_t(b) * p.Hq + hk * p.G + h0 + idx / D) * p.n_splits + split;
          p.part_o[pi * D + idx % D] = __int_as_float(0x7fc00000);
          if (idx % D == 0) p.part_m[pi] = p.part_l[pi] = __int_as_float(0x7fc00000);
        }
      }
      return;
    }
    {
      const int nxt = it + kPStages - 1;
      if (nxt < ntiles) load_tile(nxt, nxt % kPStages);
      cp_async_commit();
    }
    const uint8_t* st = stages + (it % kPStages) * L.stage;
    const uint8_t* vst = st + L.off_v;
    if (VK == V_PQ) {
      // reconstruct this tile's values as f16 rows: v[t][j*dsv + i] = cent[j][code][i]
      for (int i = threadIdx.x; i < kPRows * p.Mv; i += kPW * 32) {
        const int r = i / p.Mv, j = i % p.Mv;
        const int code = vst[r * L.v_pitch + j];
        __half* dst = reinterpret_cast<__half*>(recon + r * (D * 2 + 16)) + j * p.dsv;
        for (int e = 0; e < p.dsv; ++e)
          dst[e] = __float2half_rn(p.vcent[int64_t(j) * p.vc_sm + int64_t(code) * p.vc_sk + int64_t(e) * p.vc_sd]);
      }
      if (p.Mv * p.dsv < D)
        for (int i = threadIdx.x; i < kPRows * (D - p.Mv * p.dsv); i += kPW * 32) {
          const int r = i / (D - p.Mv * p.dsv), e = i % (D - p.Mv * p.dsv);
          reinterpret_cast<__half*>(recon + r * (D * 2 + 16))[p.Mv * p.dsv + e] = __float2half(0.f);
        }
      __syncthreads();
    }
    const int t0 = t_begin + it * kPRows + r0;
    if (t0 >= t_end) continue;

    // ---- LUT scores for tokens r0+g, r0+g+8 and heads 2hp, 2hp+1 over subspaces [jlo, jhi)
    float sc[4] = {0.f, 0.f, 0.f, 0.f};  // (row g: h0, h1), (row g+8: h0, h1)
    {
      if (p.lut_t) {
        // regrouped LUT [code][subspace][4 heads]: lane = (token lane >> 1, subspace half
        // lane & 1); step s looks up subspace 8(lane & 1) + ((s + lane) & 7) with one 16-byte
        // read of all four heads. The 16-byte unit of (code, j) sits in bank group j & 7, so
        // the 8 lanes of a quarter-warp (distinct (s + lane) & 7) never share a bank group.
        const uint2 w = *reinterpret_cast<const uint2*>(st + L.off_codes + (r0 + (lane >> 1)) * L.codes_pitch +
                                                        8 * (lane & 1));
        float2 a01 = make_float2(0.f, 0.f), a23 = make_float2(0.f, 0.f);
        const uint8_t* lb = reinterpret_cast<const uint8_t*>(lut_s);
#pragma unroll
        for (int s2 = 0; s2 < 8; ++s2) {
          // byte 0: which of the lane's 8 code bytes; byte 2: the subspace's offset j * 16
          const uint32_t r = uint32_t(s2 + lane) & 7u;
          const uint32_t rs = r | (((8u * uint32_t(lane & 1) + r) * 16u) << 16);
          const uint32_t code = prmt(w.x, w.y, rs);    // byte 0 = the code
          const uint32_t off = prmt(code, rs, 0x7706);  // [j * 16, code, 0, 0] = code * 256 + j * 16
          const float4 e = *reinterpret_cast<const float4*>(lb + off);
          a01 = add_f32x2(a01, make_float2(e.x, e.y));
          a23 = add_f32x2(a23, make_float2(e.z, e.w));
        }
        // the two subspace halves of a token are neighbouring lanes
        a01.x += __shfl_xor_sync(0xffffffffu, a01.x, 1);
        a01.y += __shfl_xor_sync(0xffffffffu, a01.y, 1);
        a23.x += __shfl_xor_sync(0xffffffffu, a23.x, 1);
        a23.y += __shfl_xor_sync(0xffffffffu, a23.y, 1);
        // into the accumulator layout: lane (g, tq) takes heads 2hp, 2hp+1 of tokens g and
        // g + 8 from lanes 2g + hp and 2g + 16 + hp (odd lanes hold heads 2, 3)
        const float2 pr = (lane & 1) ? a23 : a01;
        sc[0] = __shfl_sync(0xffffffffu, pr.x, 2 * g + hp);
        sc[1] = __shfl_sync(0xffffffffu, pr.y, 2 * g + hp);
        sc[2] = __shfl_sync(0xffffffffu, pr.x, 2 * g + 16 + hp);
        sc[3] = __shfl_sync(0xffffffffu, pr.y, 2 * g + 16 + hp);
      } else {
        const uint8_t* ca = st + L.off_codes + (r0 + g) * L.codes_pitch;
        const uint8_t* cb = st + L.off_codes + (r0 + g + 8) * L.codes_pitch;
        const float* lj = lut_s + jlo * p.K * kHC + 2 * hp;  // LUT rows of subspace j, stepped per j
        const int jstep = p.K * kHC;
        if (p.M == 16) {
          // the lane's 8 subspaces of both tokens as one 8-byte load each
          const uint2 wa = *reinterpret_cast<const uint2*>(ca + jlo), wb = *reinterpret_cast<const uint2*>(cb + jlo);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t xa = ((j < 4 ? wa.x : wa.y) >> (8 * (j & 3))) & 0xffu;
            const uint32_t xb = ((j < 4 ? wb.x : wb.y) >> (8 * (j & 3))) & 0xffu;
            const float2 a = *reinterpret_cast<const float2*>(lj + xa * kHC);
            const float2 c = *reinterpret_cast<const float2*>(lj + xb * kHC);
            sc[0] += a.x; sc[1] += a.y; sc[2] += c.x; sc[3] += c.y;
            lj += jstep;
          }
        } else {
          for (int j = jlo; j < jhi; ++j) {
            const float2 a = *reinterpret_cast<const float2*>(lj + ca[j] * kHC);
            const float2 c = *reinterpret_cast<const float2*>(lj + cb[j] * kHC);
            sc[0] += a.x; sc[1] += a.y; sc[2] += c.x; sc[3] += c.y;
            lj += jstep;
          }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[e] += __shfl_xor_sync(0xffffffffu, sc[e], 2);
      }
      if (OUTL) {
        const uint16_t* ka = reinterpret_cast<const uint16_t*>(st + L.off_kout + (r0 + g) * L.kout_pitch);
        const uint16_t* kb = reinterpret_cast<const uint16_t*>(st + L.off_kout + (r0 + g + 8) * L.kout_pitch);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float xa = ld16f(ka, c, p.ko_dtype), xb = ld16f(kb, c, p.ko_dtype);
          sc[0] = fmaf(qo[0][c], xa, sc[0]); sc[1] = fmaf(qo[1][c], xa, sc[1]);
          sc[2] = fmaf(qo[0][c], xb, sc[2]); sc[3] = fmaf(qo[1][c], xb, sc[3]);
        }
      }
    }
    const bool va = t0 + g < t_end, vb = t0 + g + 8 < t_end;
    if (VK == V_NONE) {
      if (tq < 2) {
        for (int e = 0; e < 2; ++e) {
          const int h = 2 * hp + e;
          if (h >= nheads) continue;
          float* orow = p.scores_out + int64_t(b) * p.so_sb + int64_t(hk * p.G + h0 + h) * p.so_sh;
          if (va) orow[t0 + g] = sc[e];
          if (vb) orow[t0 + g + 8] = sc[2 + e];
        }
      }
      continue;
    }

    // ---- online softmax (exp2 domain) on accumulator-layout scores. The reference mrow
    // moves only when a score passes it, to that score + kPHeadroom, so the running sums
    // are rescaled rarely and every weight 2^(x - mrow) stays <= 1.
    float pv[4];
    {
      float a[2], c[2], mx[2];
      bool grow = false;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        a[j] = va ? sc[j] * kLog2eP : -INFINITY;
        c[j] = vb ? sc[2 + j] * kLog2eP : -INFINITY;
        mx[j] = fmaxf(a[j], c[j]);
        grow |= mx[j] > mrow[j];
      }
      // the head maxima are reduced over the warp only when some score passed the reference
      if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], 4));
          mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], 8));
          mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], 16));
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float mnew = mx[j] > mrow[j] ? mx[j] + kPHeadroom : mrow[j];
          const float alpha = mrow[j] == -INFINITY ? 0.f : fast_exp2(mrow[j] - mnew);
          mrow[j] = mnew;
          lrow[j] *= alpha;
#pragma unroll
          for (int mt = 0; mt < KSTEPS; ++mt) {
            o[mt][j] *= alpha;
            o[mt][2 + j] *= alpha;
          }
          oc[j] *= alpha;
          oc[2 + j] *= alpha;
        }
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float muse = mrow[j] == -INFINITY ? 0.f : mrow[j];
        pv[j] = fast_exp2(a[j] - muse);
        pv[2 + j] = fast_exp2(c[j] - muse);
        lrow[j] += pv[j] + pv[2 + j];
      }
    }

    // ---- O^T += V^T . P^T
    if (VK == V_BF16 || VK == V_F16) {
      // 16-bit values straight from the tile; f16 values meet f16 weights
      const uint32_t pb0 = movmatrix_trans(VK == V_F16 ? pack_f16x2(pv[0], pv[1]) : pack_bf16x2(pv[0], pv[1]));
      const uint32_t pb1 = movmatrix_trans(VK == V_F16 ? pack_f16x2(pv[2], pv[3]) : pack_bf16x2(pv[2], pv[3]));
      const uint32_t vs = smem_u32(vst);
      const int vrow = r0 + (lane & 7) + (lane >> 4) * 8;
#pragma unroll
      for (int mt = 0; mt < KSTEPS; ++mt) {
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4_trans(a0, a1, a2, a3, vs + vrow * L.v_pitch + (mt * 16 + ((lane >> 3) & 1) * 8) * 2);
        if (VK == V_F16) mma_f16(o[mt], a0, a1, a2, a3, pb0, pb1);
        else mma_bf16(o[mt], a0, a1, a2, a3, pb0, pb1);
      }
    } else if (VK == V_PQ) {
      const uint32_t pb0 = movmatrix_trans(pack_f16x2(pv[0], pv[1]));
      const uint32_t pb1 = movmatrix_trans(pack_f16x2(pv[2], pv[3]));
      const uint32_t vs = smem_u32(recon);
      const int vrow = r0 + (lane & 7) + (lane >> 4) * 8;
#pragma unroll
      for (int mt = 0; mt < KSTEPS; ++mt) {
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4_trans(a0, a1, a2, a3, vs + vrow * (D * 2 + 16) + (mt * 16 + ((lane >> 3) & 1) * 8) * 2);
        mma_f16(o[mt], a0, a1, a2, a3, pb0, pb1);
      }
    } else {
      float q0 = pv[0], q1 = pv[1], q2 = pv[2], q3 = pv[3];
      if (VK == V_INT8) {
        const __half* vsr = reinterpret_cast<const __half*>(st + L.off_vs);
        const float sa = __half2float(vsr[r0 + g]), sb = __half2float(vsr[r0 + g + 8]);
        q0 *= sa; q1 *= sa; q2 *= sb; q3 *= sb;
      }
      const uint32_t pb0 = movmatrix_trans(pack_f16x2(q0, q1));
      const uint32_t pb1 = movmatrix_trans(pack_f16x2(q2, q3));
      const uint32_t vs = smem_u32(vst);
      const int vrow = r0 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int m2 = 0; m2 < KSTEPS / 2; ++m2) {
        uint32_t x0, x1, x2, x3;
        // TMA tile: 128-byte rows, 16-byte chunk c of row r at chunk c ^ (r & 7) (vrow & 7 = lane & 7)
        ldmatrix_x4_trans(x0, x1, x2, x3,
                          TMA ? vs + vrow * 128 + (((2 * m2 + (lane >> 4)) ^ (lane & 7)) << 4)
                              : vs + vrow * L.v_pitch + m2 * 32 + (lane >> 4) * 16);
        uint32_t a[8];
        const uint32_t xs[4] = {x0, x1, x2, x3};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (VK == V_FP8) {
            a[2 * u] = e4m3x2_to_f16x2(prmt(xs[u], 0, 0x0020));
            a[2 * u + 1] = e4m3x2_to_f16x2(prmt(xs[u], 0, 0x0031));
          } else {
            // int8 -> f16 halves 0x64XX, XX = x ^ 0x80: the value 1024 + x + 128 (the four
            // sign bits flipped once per word, then one byte-select PRMT per register); the
            // 1152 comes off through oc
            const uint32_t xo = xs[u] ^ 0x80808080u;
            a[2 * u] = prmt(xo, 0x64646464u, 0x4240);
            a[2 * u + 1] = prmt(xo, 0x64646464u, 0x4341);
          }
        }
        mma_f16(o[2 * m2], a[0], a[1], a[2], a[3], pb0, pb1);
        mma_f16(o[2 * m2 + 1], a[4], a[5], a[6], a[7], pb0, pb1);
      }
      if (VK == V_INT8) mma_f16(oc, 0x64806480u, 0x64806480u, 0x64806480u, 0x64806480u, pb0, pb1);
    }
  }
  if (VK == V_NONE) return;

  // ---- merge warps, write split partials
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    float l = lrow[j];
    l += __shfl_xor_sync(0xffffffffu, l, 4);
    l += __shfl_xor_sync(0xffffffffu, l, 8);
    l += __shfl_xor_sync(0xffffffffu, l, 16);
    lrow[j] = l;
  }
  cp_async_wait<0>();
  __syncthreads();
  float* red_m = reinterpret_cast<float*>(smem);  // [warps][8]
  float* red_l = red_m + kPW * 8;
  float* red_o = red_l + kPW * 8;  // [warps][4][D]
  if (g == 0) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      red_m[warp * 8 + 2 * tq + j] = mrow[j];
      red_l[warp * 8 + 2 * tq + j] = lrow[j];
    }
  }
  __syncthreads();
  if (tq < 2) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int h = 2 * tq + j;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kPW; ++w) M = fmaxf(M, red_m[w * 8 + h]);
      const float f = (M == -INFINITY) ? 0.f : exp2f(mrow[j] - M);
#pragma unroll
      for (int mt = 0; mt < KSTEPS; ++mt) {
        const bool wide = (VK == V_FP8 || VK == V_INT8);
        const int ca = wide ? mt * 16 + 2 * g : mt * 16 + g;
        const int cb = wide ? ca + 1 : ca + 8;
        // (oc is zero unless the values are int8)
        red_o[(warp * kHC + h) * D + ca] = (o[mt][j] - oc[j]) * f;
        red_o[(warp * kHC + h) * D + cb] = (o[mt][2 + j] - oc[2 + j]) * f;
      }
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < nheads * D; idx += kPW * 32) {
    const int h = idx / D, c = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kPW; ++w) M = fmaxf(M, red_m[w * 8 + h]);
    float Ls = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kPW; ++w) {
      const float f = (M == -INFINITY) ? 0.f : exp2f(red_m[w * 8 + h] - M);
      Ls += red_l[w * 8 + h] * f;
      O += red_o[(w * kHC + h) * D + c];
    }
    const int hq = hk * p.G + h0 + h;
    const int64_t pi = (int64_t(b) * p.Hq + hq) * p.n_splits + split;
    p.part_o[pi * D + c] = O;
    if (c == 0) {
      p.part_m[pi] = M * kLn2P;
      p.part_l[pi] = Ls;
    }
  }
}

// LUT[b,h,j,c] = sum_i q[b,h,j*dsub+i] * cent[j,c,i]
__global__ void pq_lut_kernel(const void* q, int q_dtype, int64_t q_sb, int64_t q_sh, int64_t q_sd, const float* cent,
                              int64_t c_sm, int64_t c_sk, int64_t c_sd, int Hq, int M, int K, int dsub, float* lut) {
  const int bh = blockIdx.y;
  const int b = bh / Hq, h = bh % Hq;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= M * K) return;
  const int j = i / K, c = i % K;
  float acc = 0.f;
  for (int e = 0; e < dsub; ++e) {
    const int64_t qo = int64_t(b) * q_sb + int64_t(h) * q_sh + int64_t(j * dsub + e) * q_sd;
    float qv;
    if (q_dtype == BD_BF16) qv = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(q)[qo]);
    else if (q_dtype == BD_F16) qv = __half2float(reinterpret_cast<const __half*>(q)[qo]);
    else qv = reinterpret_cast<const float*>(q)[qo];
    acc = fmaf(qv, cent[int64_t(j) * c_sm + int64_t(c) * c_sk + int64_t(e) * c_sd], acc);
  }
  lut[int64_t(bh) * M * K + i] = acc;
}

// codes[n, j] = argmax_c (x_h . c_h - norm_c), first index on ties: the nearest-centroid rule
// of ProductQuantizer.quantize on a CUDA device (src/quantization.py:160-199, kernel :8-60).
// x_h = x rounded to f16; c_h = the fp32 centroid rounded to x's dtype, then to f16; the
// products of f16 values are exact in fp32 and summed in fp32; norm_c = 0.5 * sum(c^2) in
// fp32, rounded to x's dtype. argmax of that score is argmin of the squared distance up to
// the f16 rounding of the operands.
__device__ __forceinline__ float round_as(float v, int dt) {
  if (dt == BD_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dt == BD_F16) return __half2float(__float2half_rn(v));
  return v;
}

__global__ void pq_encode_kernel(const void* x, int x_dtype, int64_t x_sn, const float* cent, int64_t c_sm,
                                 int64_t c_sk, int64_t c_sd, int64_t N, int M, int K, int dsub, void* codes,
                                 int codes64) {
  extern __shared__ float cs[];  // [K][dsub] f16-rounded centroids of subspace j, then [K] norms
  float* norms = cs + K * dsub;
  const int j = blockIdx.y;
  for (int i = threadIdx.x; i < K * dsub; i += blockDim.x) {
    const float c = cent[int64_t(j) * c_sm + int64_t(i / dsub) * c_sk + int64_t(i % dsub) * c_sd];
    cs[i] = __half2float(__float2half_rn(round_as(c, x_dtype)));
  }
  for (int c = threadIdx.x; c < K; c += blockDim.x) {
    float s2 = 0.f;
    for (int e = 0; e < dsub; ++e) {
      const float v = cent[int64_t(j) * c_sm + int64_t(c) * c_sk + int64_t(e) * c_sd];
      s2 = __fadd_rn(s2, __fmul_rn(v, v));
    }
    norms[c] = round_as(0.5f * s2, x_dtype);
  }
  __syncthreads();
  const int64_t n = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float xv[32];
  for (int e = 0; e < dsub; ++e) {
    const int64_t off = n * x_sn + int64_t(j) * dsub + e;
    float v;
    if (x_dtype == BD_BF16) v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[off]);
    else if (x_dtype == BD_F16) v = __half2float(reinterpret_cast<const __half*>(x)[off]);
    else v = reinterpret_cast<const float*>(x)[off];
    xv[e] = __half2float(__float2half_rn(v));
  }
  float best = -INFINITY;
  int bi = 0;
  for (int c = 0; c < K; ++c) {
    float d = 0.f;
    for (int e = 0; e < dsub; ++e) d = __fadd_rn(d, __fmul_rn(xv[e], cs[c * dsub + e]));
    const float sc = __fsub_rn(d, norms[c]);
    if (sc > best) { best = sc; bi = c; }
  }
  if (codes64) reinterpret_cast<int64_t*>(codes)[n * M + j] = bi;
  else reinterpret_cast<uint8_t*>(codes)[n * M + j] = uint8_t(bi);
}

// LUT [B,Hq,16,256] fp32 (any strides) -> one block per (batch, KV head, head chunk) of
// [256 codes][16 subspaces][4 heads], heads past the group zero. Grid (B*Hk*chunks, 16),
// 256 threads (thread = code): reads are coalesced along the codes.
__global__ void pq_lut_regroup_kernel(const float* __restrict__ lut, int64_t l_sb, int64_t l_sh, int64_t l_sm,
                                      int64_t l_sk, int Hk, int G, int head_chunks, float4* __restrict__ out) {
  // the decode kernel queued behind may start launching: it waits for this grid only
  // before it reads the regrouped LUT
  griddep_launch_dependents();
  const int bc = blockIdx.x, j = blockIdx.y, code = threadIdx.x;
  const int chunk = bc % head_chunks, bh = bc / head_chunks;
  const int hk = bh % Hk, b = bh / Hk;
  const int h0 = chunk * kHC, nheads = min(kHC, G - h0);
  float v[kHC];
#pragma unroll
  for (int h = 0; h < kHC; ++h)
    v[h] = h < nheads ? lut[int64_t(b) * l_sb + int64_t(hk * G + h0 + h) * l_sh + int64_t(j) * l_sm + int64_t(code) * l_sk]
                      : 0.f;
  out[int64_t(bc) * (256 * 16) + code * 16 + j] = make_float4(v[0], v[1], v[2], v[3]);
}

// Dynamic shared memory of one CTA (the TMA form adds its alignment slack and barriers).
inline size_t pq_cta_smem(const PqSmem& L, int D, bool tma) {
  const size_t body = size_t(L.off_stages) + size_t(kPStages) * L.stage + L.recon_bytes + (tma ? 16 + 1024 : 0);
  return std::max(body, (2 * kPW * 8 + size_t(kPW) * kHC * size_t(D)) * sizeof(float));
}

// Tensor maps of the TMA form: values [B,Hk,S,D] bytes (128-byte swizzle), codes
// [B,Hk,S,M] bytes and, for int8 values, the per-token scales [B,Hk,S] f16. Needs 16-byte
// aligned bases and strides, M a multiple of 16 stored densely, D = 128 and unit-stride scales.
bool pq_tma_maps(const PqParams& p, int vk, CUtensorMap m[3]) {
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  auto st = [](int64_t bytes, int64_t size, int64_t fallback) -> int64_t { return size > 1 ? bytes : fallback; };
  const int64_t S = p.S, Hk = p.Hk, B = p.B;
  if (p.D != 128 || (p.M % 16) || p.c_sm != 1 || !a16(p.v) || !a16(p.codes) || S <= 0) return false;
  const int64_t v_ss = p.v_ss, v_sh = st(p.v_sh, Hk, v_ss * S), v_sb = st(p.v_sb, B, v_sh * Hk);
  const int64_t c_ss = p.c_ss, c_sh = st(p.c_sh, Hk, c_ss * S), c_sb = st(p.c_sb, B, c_sh * Hk);
  for (int64_t x : {v_ss, v_sh, v_sb, c_ss, c_sh, c_sb})
    if (x <= 0 || x % 16 || x >= (int64_t(1) << 40)) return false;
  const cuuint64_t dv[4] = {128, cuuint64_t(S), cuuint64_t(Hk), cuuint64_t(B)};
  const cuuint64_t sv[3] = {cuuint64_t(v_ss), cuuint64_t(v_sh), cuuint64_t(v_sb)};
  const cuuint32_t bv[4] = {128, uint32_t(kPRows), 1, 1};
  const cuuint64_t dc[4] = {cuuint64_t(p.M), cuuint64_t(S), cuuint64_t(Hk), cuuint64_t(B)};
  const cuuint64_t sc[3] = {cuuint64_t(c_ss), cuuint64_t(c_sh), cuuint64_t(c_sb)};
  const cuuint32_t bc[4] = {uint32_t(p.M), uint32_t(kPRows), 1, 1};
  if (!encode_map(&m[0], CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, p.v, dv, sv, bv, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_map(&m[1], CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, p.codes, dc, sc, bc, CU_TENSOR_MAP_SWIZZLE_NONE))
    return false;
  if (vk == V_INT8) {
    if (p.vs_ss != 1 || !a16(p.vsc)) return false;
    const int64_t s_sh = st(p.vs_sh * 2, Hk, S * 2), s_sb = st(p.vs_sb * 2, B, s_sh * Hk);
    if (s_sh % 16 || s_sb % 16 || s_sh <= 0 || s_sb <= 0) return false;
    const cuuint64_t ds[3] = {cuuint64_t(S), cuuint64_t(Hk), cuuint64_t(B)};
    const cuuint64_t ss[2] = {cuuint64_t(s_sh), cuuint64_t(s_sb)};
    const cuuint32_t bs[3] = {uint32_t(kPRows), 1, 1};
    if (!encode_map(&m[2], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, p.vsc, ds, ss, bs, CU_TENSOR_MAP_SWIZZLE_NONE))
      return false;
  }
  return true;
}

template <int VK, bool PAGED, bool OUTL, int D, bool TMA>
int launch_pq_as(const PqParams& p, const CUtensorMap* maps, cudaStream_t st) {
  const PqSmem L = pq_smem(VK, p.M, p.K, OUTL ? p.C : 0, D, p.Mv, TMA);
  const size_t smem = pq_cta_smem(L, D, TMA);
  if (smem > 225 * 1024) return fail(BD_ERR_UNSUPPORTED, "PQ LUT too large for shared memory (M*K too big)");
  auto kern = pq_decode_kernel<VK, PAGED, OUTL, D, TMA>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    int rc = cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 225 * 1024),
                        "cudaFuncSetAttribute(pq)");
    if (rc) return rc;
    attr[dev & 63] = true;
  }
  dim3 grid(p.n_splits, p.Hk * p.head_chunks, p.B);
  if (p.lut_t)  // behind the LUT regroup: a programmatic dependent (it waits before reading the LUT)
    return launch_pdl(kern, grid, dim3(kPW * 32), smem, st, "pq_decode_kernel launch", p, maps[0], maps[1], maps[2]);
  kern<<<grid, kPW * 32, smem, st>>>(p, maps[0], maps[1], maps[2]);
  return cuda_check(cudaGetLastError(), "pq_decode_kernel launch");
}

template <int VK, bool PAGED, bool OUTL, int D>
int launch_pq(const PqParams& p, cudaStream_t st) {
  alignas(64) CUtensorMap maps[3];
  std::memset(maps, 0, sizeof maps);
  if constexpr (!PAGED && !OUTL && D == 128 && (VK == V_INT8 || VK == V_FP8)) {
    if (pq_tma_maps(p, VK, maps)) return launch_pq_as<VK, false, false, D, true>(p, maps, st);
  }
  return launch_pq_as<VK, PAGED, OUTL, D, false>(p, maps, st);
}

template <int VK, int D>
int dispatch_pq2(const PqParams& p, bool paged, bool outl, cudaStream_t st) {
  if (paged) return outl ? launch_pq<VK, true, true, D>(p, st) : launch_pq<VK, true, false, D>(p, st);
  return outl ? launch_pq<VK, false, true, D>(p, st) : launch_pq<VK, false, false, D>(p, st);
}

int dispatch_pq(const PqParams& p, int vk, bool paged, bool outl, cudaStream_t st) {
  if (p.D == 128) {
    switch (vk) {
      case V_BF16: return dispatch_pq2<V_BF16, 128>(p, paged, outl, st);
      case V_F16: return dispatch_pq2<V_F16, 128>(p, paged, outl, st);
      case V_FP8: return dispatch_pq2<V_FP8, 128>(p, paged, outl, st);
      case V_INT8: return dispatch_pq2<V_INT8, 128>(p, paged, outl, st);
      case V_PQ: return dispatch_pq2<V_PQ, 128>(p, paged, outl, st);
      default: return dispatch_pq2<V_NONE, 128>(p, paged, outl, st);
    }
  }
  switch (vk) {
    case V_BF16: return dispatch_pq2<V_BF16, 64>(p, paged, outl, st);
    case V_F16: return dispatch_pq2<V_F16, 64>(p, paged, outl, st);
    case V_FP8: return dispatch_pq2<V_FP8, 64>(p, paged, outl, st);
    case V_INT8: return dispatch_pq2<V_INT8, 64>(p, paged, outl, st);
    case V_PQ: return dispatch_pq2<V_PQ, 64>(p, paged, outl, st);
    default: return dispatch_pq2<V_NONE, 64>(p, paged, outl, st);
  }
}

}  // namespace
}  // namespace bd

namespace bd {
// host read of this file's wait-timeout counter (-1 on failure)
long long pq_wait_timeouts() {
  unsigned int v = 0;
  return cudaMemcpyFromSymbol(&v, g_pq_tma_timeouts, sizeof v) == cudaSuccess ? (long long)v : -1;
}
}  // namespace bd

extern "C" {

// Shared front end of the PQ-LUT decode entry points.
static int pq_common(const bd_tensor* lut, const bd_tensor* codes, const bd_tensor* k_out, const bd_tensor* q_out,
                     const bd_tensor* v, const bd_tensor* v_scale, const bd_tensor* v_idx, const bd_tensor* v_cent,
                     const bd_tensor* block_table, const bd_tensor* context_lens, int block_size,
                     const bd_tensor* out_or_scores, bool scores_only, void* workspace, size_t workspace_bytes,
                     bd_stream_t stream, size_t* ws_query) {
  using namespace bd;
  int rc;
  if ((rc = check_tensor(lut, "lut", 4, BD_F32)) || (rc = check_tensor(codes, "k_idx", 4, BD_U8))) return rc;
  const int64_t B = lut->shape[0], Hq = lut->shape[1], M = lut->shape[2], K = lut->shape[3];
  const int64_t Hk = codes->shape[1];
  const bool paged = block_table != nullptr;
  if (Hk <= 0 || Hq % Hk) return fail(BD_ERR_SHAPE, "H_q must be a multiple of H_k");
  if (codes->shape[3] < M) return fail(BD_ERR_SHAPE, "k_idx last dim must hold the LUT's M subspaces");
  if (K > 256 || K <= 0 || M <= 0 || M > 64) return fail(BD_ERR_UNSUPPORTED, "LUT must have M <= 64, K <= 256");
  int vk = V_NONE;
  int64_t D = 0, Mv = 0, Kv = 0, dsv = 0;
  if (!scores_only) {
    if (v_idx) {
      if ((rc = check_tensor(v_idx, "v_idx", 4, BD_U8)) || (rc = check_tensor(v_cent, "v_centroids", 3, BD_F32)))
        return rc;
      Mv = v_cent->shape[0]; Kv = v_cent->shape[1]; dsv = v_cent->shape[2];
      D = Mv * dsv;
      if (v_idx->shape[3] < Mv) return fail(BD_ERR_SHAPE, "v_idx last dim must hold M_v subspaces");
      if (Kv > 256) return fail(BD_ERR_UNSUPPORTED, "value codebooks must have <= 256 entries");
      vk = V_PQ;
    } else {
      if ((rc = check_tensor(v, "v", 4))) return rc;
      D = v->shape[3];
      if (v->dtype == BD_BF16) vk = V_BF16;
      else if (v->dtype == BD_F16) vk = V_F16;
      else if (v->dtype == BD_F8E4M3) vk = V_FP8;
      else if (v->dtype == BD_I8) {
        vk = V_INT8;
        if (!ws_query && (rc = check_tensor(v_scale, "v_scale", 3, BD_F16))) return rc;
      } else return fail(BD_ERR_DTYPE, "v must be bf16, f16, fp8 e4m3 or int8 (+ v_scale)");
      if ((rc = check_rows_aligned(v, "v"))) return rc;
    }
    if (D != 64 && D != 128) return fail(BD_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  } else {
    D = 128;
  }
  int64_t S;
  if (paged) {
    if ((rc = check_tensor(block_table, "block_table", 2, BD_I32)) ||
        (rc = check_tensor(context_lens, "context_lens", 1, BD_I32)))
      return rc;
    if (block_size <= 0 || codes->shape[2] != block_size) return fail(BD_ERR_SHAPE, "paged k_idx must be [NB,Hk,block_size,M]");
    if (block_table->shape[0] != B || context_lens->shape[0] != B) return fail(BD_ERR_SHAPE, "block_table/context_lens batch");
    S = block_table->shape[1] * block_size;
  } else {
    S = codes->shape[2];
    if (codes->shape[0] != B) return fail(BD_ERR_SHAPE, "k_idx batch must match lut");
  }
  const bool outl = k_out && k_out->ndim == 4 && k_out->shape[3] > 0;
  if (outl) {
    if ((rc = check_tensor(k_out, "k_out", 4)) || (rc = check_tensor(q_out, "q_out", 3))) return rc;
    if (k_out->shape[3] > 8) return fail(BD_ERR_UNSUPPORTED, "at most 8 outlier channels");
    if (k_out->dtype != BD_BF16 && k_out->dtype != BD_F16) return fail(BD_ERR_DTYPE, "k_out must be bf16 or f16");
    if (q_out->shape[0] != B || q_out->shape[1] != Hq || q_out->shape[2] != k_out->shape[3])
      return fail(BD_ERR_SHAPE, "q_out must be [B,Hq,C_out]");
  }
  const PqSmem Ls = pq_smem(vk, int(M), int(K), outl ? int(k_out->shape[3]) : 0, int(D), int(Mv));
  const int head_chunks = int((Hq / Hk + kHC - 1) / kHC);
  const int64_t ntiles = (S + kPRows - 1) / kPRows;
  const int64_t pairs = B * Hk * head_chunks;
  // resident CTAs per SM from the shared-memory footprint (227 KB usable per SM)
  const PqSmem Lt = pq_smem(vk, int(M), int(K), 0, int(D), int(Mv), true);
  const size_t cta_smem = std::max(pq_cta_smem(Ls, int(D), false), pq_cta_smem(Lt, int(D), true)) + 1024;
  const int64_t per_sm = std::max<int64_t>(1, std::min<int64_t>(2, int64_t(227 * 1024) / int64_t(cta_smem)));
  const int64_t slots = per_sm * num_sms();
  int64_t splits = pairs >= slots ? 1 : slots / pairs;
  splits = std::max<int64_t>(1, std::min<int64_t>(splits, std::max<int64_t>(ntiles, 1)));
  // M = 16, K = 256 (the usual codebook): the LUT is regrouped per call into the workspace
  // behind the partials, so the decode CTAs read it as one contiguous block
  const bool fast_lut = !scores_only && M == 16 && K == 256;
  const size_t part_bytes = scores_only ? 0 : partials_bytes(size_t(B * Hq), int(splits), int(D));
  const size_t lut_bytes = fast_lut ? size_t(B * Hk * head_chunks) * 256 * 16 * 16 : 0;
  const size_t need = part_bytes + (fast_lut ? lut_bytes + 256 : 0);
  if (ws_query) { *ws_query = need; return BD_OK; }
  if (!out_or_scores) return fail(BD_ERR_NULL, "output descriptor is NULL");
  if (!scores_only && (!workspace || workspace_bytes < need))
    return fail(BD_ERR_WORKSPACE, "need " + std::to_string(need) + " workspace bytes");
  PqParams p{};
  p.lut = static_cast<const float*>(lut->data);
  p.l_sb = lut->stride[0]; p.l_sh = lut->stride[1]; p.l_sm = lut->stride[2]; p.l_sk = lut->stride[3];
  p.codes = static_cast<const uint8_t*>(codes->data);
  p.c_sb = codes->stride[0]; p.c_sh = codes->stride[1]; p.c_ss = codes->stride[2]; p.c_sm = codes->stride[3];
  if (p.c_sm != 1) return fail(BD_ERR_STRIDE, "k_idx innermost dim must be contiguous");
  if (outl) {
    p.kout = static_cast<const uint16_t*>(k_out->data);
    p.ko_sb = k_out->stride[0]; p.ko_sh = k_out->stride[1]; p.ko_ss = k_out->stride[2]; p.ko_sc = k_out->stride[3];
    p.ko_dtype = k_out->dtype;
    p.qout = q_out->data; p.qo_sb = q_out->stride[0]; p.qo_sh = q_out->stride[1]; p.qo_sc = q_out->stride[2];
    p.qo_dtype = q_out->dtype;
    p.C = int(k_out->shape[3]);
  }
  if (vk == V_BF16 || vk == V_F16 || vk == V_FP8 || vk == V_INT8) {
    p.v = static_cast<const uint8_t*>(v->data); p.v_sb = v->stride[0]; p.v_sh = v->stride[1]; p.v_ss = v->stride[2];
    if (vk == V_INT8) {
      p.vsc = static_cast<const __half*>(v_scale->data);
      p.vs_sb = v_scale->stride[0]; p.vs_sh = v_scale->stride[1]; p.vs_ss = v_scale->stride[2];
    }
  } else if (vk == V_PQ) {
    p.vidx = static_cast<const uint8_t*>(v_idx->data);
    p.vi_sb = v_idx->stride[0]; p.vi_sh = v_idx->stride[1]; p.vi_ss = v_idx->stride[2]; p.vi_sm = v_idx->stride[3];
    p.vcent = static_cast<const float*>(v_cent->data);
    p.vc_sm = v_cent->stride[0]; p.vc_sk = v_cent->stride[1]; p.vc_sd = v_cent->stride[2];
    p.Mv = int(Mv); p.Kv = int(Kv); p.dsv = int(dsv);
  }
  if (paged) {
    p.btab = static_cast<const int32_t*>(block_table->data); p.bt_sb = block_table->stride[0];
    p.bt_ss = block_table->stride[1];
    p.clens = static_cast<const int32_t*>(context_lens->data);
    p.bsz = block_size;
  }
  p.B = int(B); p.Hq = int(Hq); p.Hk = int(Hk); p.G = int(Hq / Hk); p.S = int(S); p.M = int(M); p.K = int(K);
  p.D = int(D);
  p.head_chunks = head_chunks; p.ntiles = int(ntiles); p.n_splits = int(splits);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (B * Hq == 0) return BD_OK;
  if (scores_only) {
    p.scores_out = static_cast<float*>(out_or_scores->data);
    p.so_sb = out_or_scores->stride[0]; p.so_sh = out_or_scores->stride[1];
    return dispatch_pq(p, V_NONE, paged, outl, st);
  }
  Partials part = carve_partials(workspace, size_t(B * Hq), int(splits), int(D));
  p.part_m = part.m; p.part_l = part.l; p.part_o = part.o;
  if (fast_lut) {
    const uintptr_t lut_at = (reinterpret_cast<uintptr_t>(part.l + size_t(B * Hq) * splits) + 255) & ~uintptr_t(255);
    p.lut_t = reinterpret_cast<const float4*>(lut_at);
    pq_lut_regroup_kernel<<<dim3(unsigned(B * Hk * head_chunks), 16), 256, 0, st>>>(
        p.lut, p.l_sb, p.l_sh, p.l_sm, p.l_sk, int(Hk), int(Hq / Hk), head_chunks, reinterpret_cast<float4*>(lut_at));
    if ((rc = cuda_check(cudaGetLastError(), "pq_lut_regroup_kernel launch"))) return rc;
  }
  if ((rc = dispatch_pq(p, vk, paged, outl, st))) return rc;
  return launch_combine(part, int(B), int(Hq), int(D), out_or_scores, st, true);
}

size_t bd_pq_decode_workspace(const bd_tensor* lut, const bd_tensor* k_idx, const bd_tensor* v,
                              const bd_tensor* v_idx, const bd_tensor* v_centroids, const bd_tensor* block_table,
                              const bd_tensor* context_lens, int block_size) {
  size_t n = 0;
  if (pq_common(lut, k_idx, nullptr, nullptr, v, nullptr, v_idx, v_centroids, block_table, context_lens, block_size,
                nullptr, false, nullptr, 0, nullptr, &n))
    return 0;
  return n;
}

int bd_pq_decode(const bd_tensor* lut, const bd_tensor* k_idx, const bd_tensor* k_out, const bd_tensor* q_out,
                 const bd_tensor* v, const bd_tensor* v_scale, const bd_tensor* v_idx, const bd_tensor* v_centroids,
                 const bd_tensor* block_table, const bd_tensor* context_lens, int block_size, const bd_tensor* out,
                 void* workspace, size_t workspace_bytes, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if ((rc = check_tensor(out, "out", 3))) return rc;
  if (out->dtype != BD_BF16 && out->dtype != BD_F16 && out->dtype != BD_F32) return fail(BD_ERR_DTYPE, "out dtype");
  if (out->stride[2] != 1) return fail(BD_ERR_STRIDE, "out rows must be contiguous");
  return pq_common(lut, k_idx, k_out, q_out, v, v_scale, v_idx, v_centroids, block_table, context_lens, block_size,
                   out, false, workspace, workspace_bytes, stream, nullptr);
}

int bd_pq_scores(const bd_tensor* lut, const bd_tensor* k_idx, const bd_tensor* k_out, const bd_tensor* q_out,
                 const bd_tensor* scores, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if ((rc = check_tensor(scores, "scores", 3, BD_F32))) return rc;
  if (scores->stride[2] != 1) return fail(BD_ERR_STRIDE, "scores rows must be contiguous");
  if (lut && k_idx && (scores->shape[0] != lut->shape[0] || scores->shape[1] != lut->shape[1] ||
                       scores->shape[2] != k_idx->shape[2]))
    return fail(BD_ERR_SHAPE, "scores must be [B,Hq,S]");
  return pq_common(lut, k_idx, k_out, q_out, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, 0, scores, true,
                   nullptr, 0, stream, nullptr);
}

int bd_pq_build_lut(const bd_tensor* q, const bd_tensor* centroids, const bd_tensor* lut, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if ((rc = check_tensor(q, "q_rot", 3)) || (rc = check_tensor(centroids, "centroids", 3, BD_F32)) ||
      (rc = check_tensor(lut, "lut", 4, BD_F32)))
    return rc;
  const int64_t B = q->shape[0], H = q->shape[1], D = q->shape[2];
  const int64_t M = centroids->shape[0], K = centroids->shape[1], dsub = centroids->shape[2];
  if (M * dsub != D) return fail(BD_ERR_SHAPE, "centroids must be [M,K,D/M]");
  if (lut->shape[0] != B || lut->shape[1] != H || lut->shape[2] != M || lut->shape[3] != K ||
      lut->stride[3] != 1 || lut->stride[2] != K || lut->stride[1] != M * K || (B > 1 && lut->stride[0] != H * M * K))
    return fail(BD_ERR_SHAPE, "lut must be contiguous [B,H,M,K]");
  if (q->dtype != BD_BF16 && q->dtype != BD_F16 && q->dtype != BD_F32) return fail(BD_ERR_DTYPE, "q dtype");
  if (B * H * M * K == 0) return BD_OK;
  dim3 grid(unsigned((M * K + 127) / 128), unsigned(B * H));
  pq_lut_kernel<<<grid, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      q->data, q->dtype, q->stride[0], q->stride[1], q->stride[2], static_cast<const float*>(centroids->data),
      centroids->stride[0], centroids->stride[1], centroids->stride[2], int(H), int(M), int(K), int(dsub),
      static_cast<float*>(lut->data));
  return cuda_check(cudaGetLastError(), "pq_lut_kernel launch");
}

int bd_pq_encode(const bd_tensor* x, const bd_tensor* centroids, const bd_tensor* codes, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if ((rc = check_tensor(x, "x", 2)) || (rc = check_tensor(centroids, "centroids", 3, BD_F32)) ||
      (rc = check_tensor(codes, "codes", 2)))
    return rc;
  const int64_t N = x->shape[0], D = x->shape[1];
  const int64_t M = centroids->shape[0], K = centroids->shape[1], dsub = centroids->shape[2];
  if (M * dsub != D) return fail(BD_ERR_SHAPE, "centroids must be [M,K,D/M]");
  if (dsub > 32) return fail(BD_ERR_UNSUPPORTED, "sub-vector length must be <= 32");
  if (codes->dtype != BD_U8 && codes->dtype != BD_I64) return fail(BD_ERR_DTYPE, "codes must be uint8 or int64");
  if (codes->dtype == BD_U8 && K > 256) return fail(BD_ERR_VALUE, "uint8 codes need K <= 256");
  if (codes->shape[0] != N || codes->shape[1] != M || codes->stride[1] != 1 || (N > 1 && codes->stride[0] != M))
    return fail(BD_ERR_SHAPE, "codes must be contiguous [N,M]");
  if (x->stride[1] != 1) return fail(BD_ERR_STRIDE, "x rows must be contiguous");
  if (x->dtype != BD_BF16 && x->dtype != BD_F16 && x->dtype != BD_F32) return fail(BD_ERR_DTYPE, "x dtype");
  const size_t smem = size_t(K * (dsub + 1)) * sizeof(float);
  if (smem > 200 * 1024) return fail(BD_ERR_UNSUPPORTED, "codebook too large");
  if (N * M == 0) return BD_OK;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    if ((rc = cuda_check(cudaFuncSetAttribute(pq_encode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024),
                         "cudaFuncSetAttribute(pq_encode)")))
      return rc;
    attr[dev & 63] = true;
  }
  dim3 grid(unsigned((N + 127) / 128), unsigned(M));
  pq_encode_kernel<<<grid, 128, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      x->data, x->dtype, x->stride[0], static_cast<const float*>(centroids->data), centroids->stride[0],
      centroids->stride[1], centroids->stride[2], N, int(M), int(K), int(dsub), codes->data, codes->dtype == BD_I64);
  return cuda_check(cudaGetLastError(), "pq_encode_kernel launch");
}

}  // extern "C"
