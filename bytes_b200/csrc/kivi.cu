// KIVI-style 2/4-bit KV-cache decode attention, the KIVI pack step and the KIVI GEMV.
//
// Reference contract (saifmb0/bytes, benchmarks/kivi_latency.py:26-90):
//   Kq  int32 [B,Hk,D,Sq/fpi]  keys quantised per channel over groups of 32 tokens,
//                              token e of a channel row at word e/fpi, bits (e%fpi)*bits
//   Ks,Km f16 [B,Hk,D,Sq/32]   per (channel, token-group) scale and minimum
//   Vq  int32 [B,Hk,Sq,D/fpi]  values quantised per token over groups of 32 channels
//   Vs,Vm f16 [B,Hk,Sq,D/32]
//   K_res,V_res bf16 [B,Hk,R,D] the most recent R tokens at full precision
//   out = softmax(Q.[K;K_res]^T / sqrt(D)) . [V;V_res]          (fpi = 32/bits)
//
// Fused decode design (one CTA = (batch, KV head, head chunk of 8, token split)):
//  * A 128-token tile of codes, scales and minima streams into shared memory through a
//    cp.async pipeline; each of the 4 warps owns 32 tokens = one key group.
//  * Keys: score = sum_c q_c (code*s_c + m_c) = sum_c (q_c s_c) code + sum_c q_c m_c.
//    The scale folds into Q' = q*s (f16, HMUL2 per warp per group), so the contraction
//    runs on the tensor cores over raw codes: S^T[16 tok x 8 heads] += codes . Q'^T
//    (mma.sync m16n8k16 f16 -> f32); the per-(head, group) bias sum_c q_c m_c is one
//    more MMA with the group's minima in every A row, so each lane reads its heads' bias
//    straight from its own accumulators.
//  * Codes become MMA operands in registers with no shared-memory staging of unpacked
//    data: a 2-bit (4-bit) field masked into the low byte of an f16 is the exact
//    subnormal code * 2^(pos-24). One byte-select PRMT of two packed words puts the
//    right byte of each into the two halves of an operand register and one AND keeps
//    the field, so every register (two codes) costs two ALU ops. The field position
//    depends only on the accumulator row a lane owns, so 2^(24-pos) is a per-lane
//    constant applied to the fp32 accumulators.
//  * Values: O^T[16 ch x 8 heads] += codes^T[16 ch x 16 tok] . P'^T[16 tok x 8], with the
//    per-token scale folded into P' = P*s_v (one version per 32-channel group); the
//    minima contribute sum_t P_t m_t per (group, head), again one MMA per row block.
//  * Row/token permutations are chosen so every shared-memory read is conflict-free
//    and the movmatrix transpose of P lands directly in the PV operand layout.
//  * The bf16 residual window runs through the dense decode kernel in its merge mode,
//    launched as a programmatic dependent of this grid: one window CTA per (batch, KV
//    head, head chunk) attends the window, waits for this grid, then merges the group's
//    split slots and the window partial into the output itself (no combine kernel).
//    When the window needs several CTAs per group, a log-sum-exp combine follows instead.
//  * Splits are balanced to one wave of 3 or 4 CTAs per SM (split s owns tiles
//    [s*T/n, (s+1)*T/n)), so no SM carries a second round.
#include "common.cuh"
#include "decode_shared.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>

namespace bd {
namespace {

constexpr int kWarpsK = 4;
constexpr int kTile = 128;  // tokens per tile
constexpr int kStagesK = 2;
constexpr float kLog2eK = 1.4426950408889634f;
constexpr float kLn2K = 0.6931471805599453f;
constexpr int kRedPitch = 132;  // floats per head row of the epilogue buffer (padded: no bank conflicts)
constexpr int kKChunk = 4;      // tiles per key scale/min chunk

// Shared-memory layout. Key tile: TMA (2-bit only) lands it unpadded with the 32-byte
// swizzle (16-byte chunk c of row r at chunk c ^ ((r >> 2) & 1)); the cp.async form pads
// rows to 48 / 80 bytes instead. 2-bit value tile: token t of the tile sits at row
// (t & 7) * 16 + (t >> 3) (32-byte rows), so the four tokens that the four lane columns of
// a warp read at once fall in four different bank groups; the 4-bit value tile keeps
// token order in padded 80-byte rows.
template <int BITS, bool TMA = false>
struct KL {
  static constexpr int FPI = 32 / BITS;
  static constexpr int KQ_WORDS = kTile / FPI;          // words per channel per tile
  static constexpr int KQ_PITCH = TMA ? 32 : (BITS == 2 ? 48 : 80);  // smem bytes per channel row
  static constexpr int VQ_WORDS = 128 / FPI;            // words per token (D = 128)
  static constexpr int VQ_PITCH = BITS == 2 ? 32 : 80;
  static constexpr int KQ_BYTES = 128 * KQ_PITCH;
  static constexpr int VQ_BYTES = kTile * VQ_PITCH;
  static constexpr int VS_BYTES = kTile * 8;  // 4 groups x f16 per token
  static constexpr int OFF_VQ = KQ_BYTES;
  static constexpr int OFF_VS = OFF_VQ + VQ_BYTES;
  static constexpr int OFF_VM = OFF_VS + VS_BYTES;
  static constexpr int STAGE = OFF_VM + VS_BYTES;
  // Key scales/minima arrive per chunk of kKChunk tiles (16 groups = 32 contiguous bytes
  // of each channel row), double-buffered: [2 buffers][scale, min][128 ch][16 groups] f16.
  // A warp's copy instruction then covers 8 channel rows instead of 32.
  static constexpr int KC_ROW = 4 * kKChunk * 2;  // bytes per channel row of one chunk
  static constexpr int KC_BYTES = 2 * 128 * KC_ROW;
  static constexpr int OFF_KC = kStagesK * STAGE;
  // Key scale/min of the current tile regrouped per lane column: [scale g0..g3, min g0..g3]
  // x [4 columns tq, 80-byte pitch] x 32 f16; channel 16j + 8h + 2tq + l sits in 16-byte
  // unit j >> 1 at u32 slot 2h + (j & 1), half l, so one 16-byte read gives a lane the
  // operands of k-steps j = 2k and 2k+1 in MMA register order
  static constexpr int T_COL = 80;
  static constexpr int T_GROUP = 4 * T_COL;
  static constexpr int T_BYTES = 8 * T_GROUP;
  static constexpr int OFF_T = OFF_KC + 2 * KC_BYTES;  // two buffers: tile it and tile it + 1
  // 2-bit: each warp's value scales / minima of its 32 tokens as (token, token + 4) operand
  // pairs: [scale, min][4 groups][4 lane columns tq][(rb, e) = 4 pairs] half2
  static constexpr int VP_WARP = 2 * 4 * 4 * 4 * 4;
  static constexpr int OFF_VP = OFF_T + 2 * T_BYTES;
  static constexpr int OFF_BAR = OFF_VP + (BITS == 2 ? 4 * VP_WARP : 0);  // TMA: one mbarrier per stage
  static constexpr int SMEM = OFF_BAR + kStagesK * 8;
  static constexpr uint32_t TMA_BYTES = 128 * 32 + kTile * 32 + 2 * kTile * 8;  // K, V codes, V scale, V min
  static_assert(!TMA || (BITS == 2 && STAGE % 1024 == 0), "TMA stages hold the 2-bit tile at 1024-byte alignment");
};

// Byte offset of (token t, 16-byte chunk c) in the 2-bit value tile.
__host__ __device__ constexpr int vq2_offset(int t, int c) { return ((t & 7) * 16 + (t >> 3)) * 32 + c * 16; }

struct KiviParams {
  const void* q; int64_t q_sb, q_sh; int q_dtype;
  const uint32_t* kq; int64_t kq_sb, kq_sh, kq_sc;
  const __half* ks; int64_t ks_sb, ks_sh, ks_sc;
  const __half* km; int64_t km_sb, km_sh, km_sc;
  const uint32_t* vq; int64_t vq_sb, vq_sh, vq_st;
  const __half* vs; int64_t vs_sb, vs_sh, vs_st;
  const __half* vm; int64_t vm_sb, vm_sh, vm_st;
  int B, Hq, Hk, G, Sq;
  int head_chunks;
  int nsplit, ntiles;  // split s owns tiles [s*ntiles/nsplit, (s+1)*ntiles/nsplit)
  float scale_log2;
  float* part_m; float* part_l; float* part_o; int split_stride;
};

__device__ __forceinline__ float load_qk(const KiviParams& p, int64_t off) {
  switch (p.q_dtype) {
    case BD_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.q)[off]);
    case BD_F16: return __half2float(reinterpret_cast<const __half*>(p.q)[off]);
    default: return reinterpret_cast<const float*>(p.q)[off];
  }
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
__device__ __forceinline__ uint32_t lds_u32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t lds_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

// TMA waits that ran past their iteration limit (the kernel then carries on with
// whatever landed; a non-zero count means a result of that launch is wrong)
__device__ unsigned int g_kivi_tma_timeouts = 0;

// Headroom of the lazily rescaled softmax reference: when a tile's maximum exceeds the
// reference, the reference moves to that maximum + kHeadroom (log2 units), so the running
// sums are rescaled only when a score beats the last maximum by more than 2^kHeadroom and
// every weight 2^(x - reference) stays <= 1.
constexpr float kHeadroom = 4.f;

template <int BITS, bool TMA, int MINB>
__global__ void __launch_bounds__(kWarpsK * 32, MINB)
    kivi_decode_kernel(const KiviParams p, const __grid_constant__ CUtensorMap tm_kq,
                       const __grid_constant__ CUtensorMap tm_vq, const __grid_constant__ CUtensorMap tm_vs,
                       const __grid_constant__ CUtensorMap tm_vm) {
  using L = KL<BITS, TMA>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // TMA destinations must sit on the swizzle atom: align the working base by hand (the
  // launch adds 1 KB); every shared-memory access below goes through `smem`
  uint8_t* smem = TMA ? smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u) : smem_raw;
  uint8_t* tsm = smem + L::OFF_T;  // key scale / min per lane column, buffer tile & 1
  const uint32_t bar0 = smem_u32(smem + L::OFF_BAR);
  if (TMA) {
    if (threadIdx.x == 0) {
      for (int s = 0; s < kStagesK; ++s) mbar_init(bar0 + 8 * s, 1);
      mbar_fence_init();
    }
    __syncthreads();
  }
  // the residual-window kernel queued behind this one reads nothing this grid writes
  griddep_launch_dependents();
  const int split = blockIdx.x;
  const int hk = blockIdx.y / p.head_chunks;
  const int chunk = blockIdx.y % p.head_chunks;
  const int b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int tile0 = int(int64_t(split) * p.ntiles / p.nsplit);
  const int ntiles = int(int64_t(split + 1) * p.ntiles / p.nsplit) - tile0;
  const int t_begin = tile0 * kTile;
  const int t_end = min(p.Sq, t_begin + ntiles * kTile);
  const int h0 = chunk * 8;
  const int nheads = min(8, p.G - h0);
  // Lane roles. A 2-bit (4-bit) field masked into the low byte of an f16 half is the exact
  // subnormal code * 2^(pos - 24); the power of two is undone on the fp32 accumulators.
  //  2-bit: lane g owns byte g & 3 of word g >> 2 of the warp's 32-token key group, i.e.
  //   tokens 16(g>>2) + 4(g&3) + {0,1,2,3}; QK accumulator row g (g+8) of row block rb
  //   takes field 2rb (2rb+1) of that byte, so one byte-select PRMT of two channel words
  //   feeds four operand registers (one AND each). On the value side m-tile pair i
  //   (channels 32i..32i+31, one scale group) gives lane g byte g & 3 of word 2i + (g>>2):
  //   row g (g+8) of m-tile 2i+e is channel 16(2i + (g>>2)) + 4(g&3) + 2e (+1).
  //  4-bit: row g (g+8) of a row block is token rho (rho+8), rho = (g>>1) + 4(g&1), with
  //   one PRMT per operand register; value row g (g+8) of m-tile mt is channel 16mt+g (+8).
  const int rho = (g >> 1) + 4 * (g & 1);
  // Byte-select PRMT selectors: byte x of the first word -> result byte 0 and byte x of
  // the second word -> result byte 2 (bytes 1 and 3 are masked off afterwards).
  uint32_t selK0, selK1, mskK, selV0, mskV;
  float subK, subV;
  if (BITS == 2) {
    selK0 = selK1 = selV0 = uint32_t(g & 3) | (uint32_t(4 + (g & 3)) << 8);
    mskK = mskV = 0u;  // fields are compile-time: 0x00030003 << 2 * pos
    subK = subV = 0.f;
  } else {
    selK0 = selK1 = uint32_t(rho >> 1) | (uint32_t(4 + (rho >> 1)) << 8);
    mskK = 0x000F000Fu << (4 * (rho & 1));
    subK = __int_as_float((127 + 24 - 4 * (rho & 1)) << 23);
    selV0 = uint32_t(g >> 1) | (uint32_t(4 + (g >> 1)) << 8);
    mskV = 0x000F000Fu << (4 * (g & 1));
    subV = __int_as_float((127 + 24 - 4 * (g & 1)) << 23);
  }
  (void)selK1;

  const uint32_t* kq_base = p.kq + int64_t(b) * p.kq_sb + int64_t(hk) * p.kq_sh;
  const __half* ks_base = p.ks + int64_t(b) * p.ks_sb + int64_t(hk) * p.ks_sh;
  const __half* km_base = p.km + int64_t(b) * p.km_sb + int64_t(hk) * p.km_sh;
  const uint32_t* vq_base = p.vq + int64_t(b) * p.vq_sb + int64_t(hk) * p.vq_sh;
  const __half* vs_base = p.vs + int64_t(b) * p.vs_sb + int64_t(hk) * p.vs_sh;
  const __half* vm_base = p.vm + int64_t(b) * p.vm_sb + int64_t(hk) * p.vm_sh;

  // Global -> shared copy assignment of this thread, fixed over the split's tiles.
  constexpr int NCH = L::KQ_WORDS / 4;  // 16-byte key chunks per channel row (2 or 4)
  constexpr int NVC = L::VQ_WORDS / 4;  // 16-byte value chunks per token row (2 or 4)
  const int k_row = threadIdx.x / NCH, k_ck = threadIdx.x % NCH;
  const int v_row = threadIdx.x / NVC, v_ck = threadIdx.x % NVC;
  const uint32_t* k_src = kq_base + int64_t(k_row) * p.kq_sc + t_begin / L::FPI + k_ck * 4;
  const uint32_t* v_src = vq_base + int64_t(t_begin + v_row) * p.vq_st + v_ck * 4;
  // key scale/min chunks: thread = (channel row kc_row + 32i, 8-byte piece kc_piece)
  const int kc_row = threadIdx.x >> 2, kc_piece = threadIdx.x & 3;
  const __half* ks_src = ks_base + int64_t(kc_row) * p.ks_sc + t_begin / 32 + 4 * kc_piece;
  const __half* km_src = km_base + int64_t(kc_row) * p.km_sc + t_begin / 32 + 4 * kc_piece;
  const int64_t ks_pass = 32 * p.ks_sc, km_pass = 32 * p.km_sc;
  const int groups_end = (t_end + 31) / 32;  // first group index past the split
  const uint32_t kc_dst = smem_u32(smem + L::OFF_KC) + kc_row * L::KC_ROW + kc_piece * 8;
  const __half* vs_src = vs_base + int64_t(t_begin + threadIdx.x) * p.vs_st;
  const __half* vm_src = vm_base + int64_t(t_begin + threadIdx.x) * p.vm_st;
  const int64_t k_pass = int64_t(128 / NCH) * p.kq_sc;  // channel rows per pass of the CTA
  const int64_t v_pass = int64_t(128 / NVC) * p.vq_st;
  const uint32_t k_dst = k_row * L::KQ_PITCH + k_ck * 16;
  // value rows per pass: 64 tokens (2-bit: +8 row slots of the interleaved tile) or 32
  const uint32_t v_dst = L::OFF_VQ + (BITS == 2 ? vq2_offset(v_row, v_ck) : v_row * L::VQ_PITCH + v_ck * 16);
  constexpr uint32_t V_PASS_BYTES = BITS == 2 ? 8 * 32 : (128 / NVC) * L::VQ_PITCH;
  auto load_tile = [&](int tile, int stage) {
    const int t0 = t_begin + tile * kTile;
    const uint32_t sbase = smem_u32(smem + stage * L::STAGE);
    const int64_t vt = int64_t(tile) * kTile;
    if (TMA) {
      // one thread moves the whole tile; rows past the sequence end arrive as zeros
      if (threadIdx.x == 0) {
        const uint32_t bar = bar0 + 8 * stage;
        mbar_arrive_expect_tx(bar, L::TMA_BYTES);
        tma_load_4d(sbase, &tm_kq, t0 / L::FPI, 0, hk, b, bar);
        // value map dims {word, token / 8, token % 8, head, batch}: the box lands in the
        // interleaved row order of the 2-bit value tile
        tma_load_5d(sbase + L::OFF_VQ, &tm_vq, 0, t0 / 8, 0, hk, b, bar);
        tma_load_4d(sbase + L::OFF_VS, &tm_vs, 0, t0 / 2, hk, b, bar);
        tma_load_4d(sbase + L::OFF_VM, &tm_vm, 0, t0 / 2, hk, b, bar);
      }
    } else if (t0 + kTile <= t_end) {
#pragma unroll
      for (int i = 0; i < NCH; ++i)
        cp_async16(sbase + k_dst + i * (128 / NCH) * L::KQ_PITCH, k_src + i * k_pass + tile * L::KQ_WORDS, 16);
#pragma unroll
      for (int i = 0; i < NVC; ++i)
        cp_async16(sbase + v_dst + i * V_PASS_BYTES, v_src + i * v_pass + vt * p.vq_st, 16);
      cp_async8(sbase + L::OFF_VS + threadIdx.x * 8, vs_src + vt * p.vs_st, 8);
      cp_async8(sbase + L::OFF_VM + threadIdx.x * 8, vm_src + vt * p.vm_st, 8);
    } else {
      // last, partial tile of the sequence: zero-fill past t_end (src-size 0 reads nothing)
      const int words_left = (t_end - t0 + L::FPI - 1) / L::FPI - k_ck * 4;
      const int kv = max(0, min(4, words_left));
#pragma unroll
      for (int i = 0; i < NCH; ++i)
        cp_async16(sbase + k_dst + i * (128 / NCH) * L::KQ_PITCH,
                   kv ? k_src + i * k_pass + tile * L::KQ_WORDS : k_src, kv * 4);
#pragma unroll
      for (int i = 0; i < NVC; ++i) {
        const bool ok = t0 + v_row + i * (128 / NVC) < t_end;
        cp_async16(sbase + v_dst + i * V_PASS_BYTES, ok ? v_src + i * v_pass + vt * p.vq_st : v_src, ok ? 16 : 0);
      }
      const bool ok = t0 + int(threadIdx.x) < t_end;
      cp_async8(sbase + L::OFF_VS + threadIdx.x * 8, ok ? vs_src + vt * p.vs_st : vs_base, ok ? 8 : 0);
      cp_async8(sbase + L::OFF_VM + threadIdx.x * 8, ok ? vm_src + vt * p.vm_st : vm_base, ok ? 8 : 0);
    }
  };
  // key scale/min of tiles [tile, tile + kKChunk) (16 groups per channel row) into chunk
  // buffer (tile / kKChunk) & 1
  auto load_chunk = [&](int tile) {
    const uint32_t dst = kc_dst + ((tile / kKChunk) & 1) * L::KC_BYTES;
    const int goff = tile * 4 + 4 * kc_piece;  // first group of this piece, relative to t_begin
    const int gv = max(0, min(4, groups_end - (t_begin / 32 + goff)));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      cp_async8(dst + i * 32 * L::KC_ROW, gv ? ks_src + i * ks_pass + tile * 4 : ks_base, gv * 2);
      cp_async8(dst + 128 * L::KC_ROW + i * 32 * L::KC_ROW, gv ? km_src + i * km_pass + tile * 4 : km_base, gv * 2);
    }
  };

  float o[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  float cacc[4] = {0.f, 0.f, 0.f, 0.f};  // rows g<4: sum_t P_t * m_v[t][group g], heads 2tq,2tq+1
  float mref[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};

  // this thread's slot in the per-column key scale layout (thread = channel)
  const uint32_t t_slot = ((threadIdx.x >> 1) & 3) * L::T_COL + (threadIdx.x >> 5) * 16 +
                          (((threadIdx.x >> 3) & 1) * 2 + ((threadIdx.x >> 4) & 1)) * 4 + (threadIdx.x & 1) * 2;
  // 2-bit value reads: row block (tq + 4 warp) of the interleaved tile, word g >> 2
  const uint32_t v_lane = (tq + 4 * warp) * 32 + 4 * (g >> 2);

  // key scale/min of tile `tile`, regrouped per lane column into buffer tile & 1 (one
  // channel per thread); reads a chunk that every thread's copies filled
  auto regroup = [&](int tile) {
    const uint8_t* kc = smem + L::OFF_KC + ((tile / kKChunk) & 1) * L::KC_BYTES + threadIdx.x * L::KC_ROW +
                        (tile % kKChunk) * 8;
    const uint2 s4 = *reinterpret_cast<const uint2*>(kc);
    uint8_t* ts = tsm + (tile & 1) * L::T_BYTES + t_slot;
    *reinterpret_cast<uint16_t*>(ts + 0 * L::T_GROUP) = uint16_t(s4.x);
    *reinterpret_cast<uint16_t*>(ts + 1 * L::T_GROUP) = uint16_t(s4.x >> 16);
    *reinterpret_cast<uint16_t*>(ts + 2 * L::T_GROUP) = uint16_t(s4.y);
    *reinterpret_cast<uint16_t*>(ts + 3 * L::T_GROUP) = uint16_t(s4.y >> 16);
  };
  // ldmatrix.trans rows of a chunk's key minima for the per-chunk bias MMA: matrix lane >> 3
  // = (channel half lane >> 4, group half (lane >> 3) & 1)
  const uint32_t lm_off = uint32_t(((lane >> 4) * 8 + (lane & 7)) * L::KC_ROW + ((lane >> 3) & 1) * 16);
  float bacc[4] = {0.f, 0.f, 0.f, 0.f};  // key bias of the chunk's 16 groups (rows), heads 2tq, 2tq+1
  // 2-bit: this lane's slot in its warp's value operand pairs (lane = token 32 warp + lane)
  uint8_t* vp_warp = smem + L::OFF_VP + warp * L::VP_WARP;
  const uint32_t vp_tok = ((((lane >> 3) * 4 + ((lane & 7) >> 1 & 1) * 2 + (lane & 1)) * 4) + ((lane & 7) >> 2) * 2);

  // prologue: tile 0 and the first key scale/min chunk in flight
  if (ntiles > 0) {
    load_tile(0, 0);
    load_chunk(0);
  }
  cp_async_commit();

  // the query loads follow the first tile copies, so their latencies overlap
  // query of head g as f16 pairs in MMA k order: qh[j][0] = channels 16j+2tq,+1;
  // qh[j][1] = 16j+8+2tq,+1. A power-of-two pre-scale keeps |q| <= 2^8 in f16.
  uint32_t qh[8][2];
  float score_mul = p.scale_log2;
  {
    const bool ok = g < nheads;
    const int64_t qoff = int64_t(b) * p.q_sb + int64_t(hk * p.G + h0 + (ok ? g : 0)) * p.q_sh;
    float qv[8][4];
    float amax = 0.f;
    // channel pairs (2tq, 2tq+1) are adjacent: one 32-bit load per pair for 16-bit queries
    // whose rows start on an even element (the common case), element loads otherwise
    const bool pairs = p.q_dtype != BD_F32 && ((qoff & 1) == 0) && ((reinterpret_cast<uintptr_t>(p.q) & 3) == 0);
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int64_t off = qoff + 16 * j + 2 * tq + (e >> 1) * 8;
        float2 v = make_float2(0.f, 0.f);
        if (ok && pairs) {
          const uint32_t w = *reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint16_t*>(p.q) + off);
          v = p.q_dtype == BD_BF16 ? __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w))
                                   : __half22float2(*reinterpret_cast<const __half2*>(&w));
        } else if (ok) {
          v = make_float2(load_qk(p, off), load_qk(p, off + 1));
        }
        qv[j][e] = v.x;
        qv[j][e + 1] = v.y;
        amax = fmaxf(amax, fmaxf(fabsf(v.x), fabsf(v.y)));
      }
    amax = warp_max(amax);
    int ex = 0;
    frexpf(amax, &ex);
    const int shift = ex > 8 ? ex - 8 : 0;
    const float qs = ldexpf(1.f, -shift);
    score_mul = ldexpf(p.scale_log2, shift);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      qh[j][0] = pack_f16x2(qv[j][0] * qs, qv[j][1] * qs);
      qh[j][1] = pack_f16x2(qv[j][2] * qs, qv[j][3] * qs);
    }
  }

  // accumulator -> log2-domain score: kmul[2rb + h] for row g + 8h of row block rb
  float kmul[4];
#pragma unroll
  for (int f = 0; f < 4; ++f)
    kmul[f] = BITS == 2 ? __int_as_float((127 + 24 - 2 * f) << 23) * score_mul : subK * score_mul;


  // tile 0's key scale/min regrouped before the loop; each iteration regroups the next
  // tile's while this one computes, so one barrier per tile orders both buffers
  cp_async_wait<0>();
  __syncthreads();
  if (ntiles > 0) regroup(0);

  for (int it = 0; it < ntiles; ++it) {
    // cp.async groups (one committed per iteration): without TMA this tile's copies, the
    // last group; with TMA only the key scale/min chunks, and the one regroup(it + 1)
    // reads below was committed three iterations ago, so the two newest may stay pending
    if (TMA) cp_async_wait<2>();
    else cp_async_wait<0>();
    const bool lost = TMA && !mbar_wait(bar0 + 8 * (it % kStagesK), (it / kStagesK) & 1);
    // this tile landed, the regrouped scales of this tile are visible, and every thread is
    // done with the previous tile's stage and scale buffer
    if (__syncthreads_or(lost)) {
      // a tile copy never completed: give it one more bounded wait (no copy may land in
      // shared memory after this CTA exits), mark this CTA's partials as failed (NaN, so
      // the merged output is NaN) and count the event for bd_wait_timeouts()
      if (threadIdx.x == 0) atomicAdd(&g_kivi_tma_timeouts, 1u);
      mbar_wait(bar0 + 8 * (it % kStagesK), (it / kStagesK) & 1);
      cp_async_wait<0>();
      const int64_t pi0 = (int64_t(b) * p.Hq + hk * p.G + h0) * p.split_stride + split;
      for (int i = threadIdx.x; i < nheads * 128; i += kWarpsK * 32) {
        const int64_t pi = pi0 + int64_t(i >> 7) * p.split_stride;
        p.part_o[pi * 128 + (i & 127)] = __int_as_float(0x7fc00000);
        if ((i & 127) == 0) p.part_m[pi] = p.part_l[pi] = __int_as_float(0x7fc00000);
      }
      return;
    }
    if (it + 1 < ntiles) load_tile(it + 1, (it + 1) % kStagesK);
    // the chunk after next, into the buffer whose last reader was the regroup of tile it
    if (it % kKChunk == 0 && it + kKChunk < ntiles) load_chunk(it + kKChunk);
    cp_async_commit();
    if (it + 1 < ntiles) regroup(it + 1);
    const uint8_t* st = smem + (it % kStagesK) * L::STAGE;
    const uint8_t* tsc = tsm + (it & 1) * L::T_BYTES;
    const int tb = t_begin + it * kTile + 32 * warp;  // first token of this warp's group
    if (tb >= t_end) continue;

    // ---- key bias sum_c q_c m_c of all 16 groups of a 4-tile chunk, once per chunk: the
    // chunk's minima [16 groups x 16 channels] per k-step are the A operand (ldmatrix.trans
    // of the channel-major chunk buffer), accumulator rows = groups, columns = heads
    if (it % kKChunk == 0) {
      const uint32_t mb =
          smem_u32(smem + L::OFF_KC + ((it / kKChunk) & 1) * L::KC_BYTES + 128 * L::KC_ROW) + lm_off;
      bacc[0] = bacc[1] = bacc[2] = bacc[3] = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4_trans(a0, a1, a2, a3, mb + 16 * j * L::KC_ROW);
        mma_f16(bacc, a0, a1, a2, a3, qh[j][0], qh[j][1]);
      }
    }
    float bias[2];
    {
      const int r = 4 * (it % kKChunk) + warp;  // this warp's group within the chunk
      const int src = ((r & 7) << 2) | tq;
      bias[0] = __shfl_sync(0xffffffffu, r < 8 ? bacc[0] : bacc[2], src) * score_mul;
      bias[1] = __shfl_sync(0xffffffffu, r < 8 ? bacc[1] : bacc[3], src) * score_mul;
    }
    // ---- Q' = q * s_k (f16) from the regrouped key scales
    uint32_t qb[8][2];
    {
      const uint4* tsr = reinterpret_cast<const uint4*>(tsc + warp * L::T_GROUP + tq * L::T_COL);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint4 sc = tsr[k];
        qb[2 * k][0] = h2u(__hmul2(u2h(qh[2 * k][0]), u2h(sc.x)));
        qb[2 * k][1] = h2u(__hmul2(u2h(qh[2 * k][1]), u2h(sc.z)));
        qb[2 * k + 1][0] = h2u(__hmul2(u2h(qh[2 * k + 1][0]), u2h(sc.y)));
        qb[2 * k + 1][1] = h2u(__hmul2(u2h(qh[2 * k + 1][1]), u2h(sc.w)));
      }
    }

    // ---- S^T (each row scaled by 2^(pos-24)) for the warp's two 16-token row blocks
    float s[2][4];
#pragma unroll
    for (int rb = 0; rb < 2; ++rb) s[rb][0] = s[rb][1] = s[rb][2] = s[rb][3] = 0.f;
    // rows 2tq + {0, 1, 8, 9} (+16j) share the 32-byte swizzle bit (row >> 2) & 1 = tq >> 1
    const uint8_t* kst = st + (2 * tq) * L::KQ_PITCH +
                         (TMA ? ((((warp >> 1) ^ (tq >> 1)) << 4) + (warp & 1) * 8) : warp * (BITS == 2 ? 8 : 16));
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      // channels c0, c0+1 (k = 2tq, 2tq+1) and c0+8, c0+9 (k = 2tq+8, 2tq+9)
      const uint8_t* kr = kst + 16 * j * L::KQ_PITCH;
      if (BITS == 2) {
        // this lane's word (tokens 0..15 or 16..31 of the group) of the four channel rows
        const uint8_t* kw = kr + 4 * (g >> 2);
        const uint32_t rab = prmt(lds_u32(kw), lds_u32(kw + L::KQ_PITCH), selK0);
        const uint32_t rcd = prmt(lds_u32(kw + 8 * L::KQ_PITCH), lds_u32(kw + 9 * L::KQ_PITCH), selK0);
        mma_f16(s[0], rab & 0x00030003u, rab & 0x000C000Cu, rcd & 0x00030003u, rcd & 0x000C000Cu, qb[j][0], qb[j][1]);
        mma_f16(s[1], rab & 0x00300030u, rab & 0x00C000C0u, rcd & 0x00300030u, rcd & 0x00C000C0u, qb[j][0], qb[j][1]);
      } else {
        // .x/.y = tokens 0..7 / 8..15 (row block 0), .z/.w = tokens 16..23 / 24..31
        const uint4 wa = *reinterpret_cast<const uint4*>(kr);
        const uint4 wb = *reinterpret_cast<const uint4*>(kr + L::KQ_PITCH);
        const uint4 wc = *reinterpret_cast<const uint4*>(kr + 8 * L::KQ_PITCH);
        const uint4 wd = *reinterpret_cast<const uint4*>(kr + 9 * L::KQ_PITCH);
        mma_f16(s[0], prmt(wa.x, wb.x, selK0) & mskK, prmt(wa.y, wb.y, selK0) & mskK,
                prmt(wc.x, wd.x, selK0) & mskK, prmt(wc.y, wd.y, selK0) & mskK, qb[j][0], qb[j][1]);
        mma_f16(s[1], prmt(wa.z, wb.z, selK0) & mskK, prmt(wa.w, wb.w, selK0) & mskK,
                prmt(wc.z, wd.z, selK0) & mskK, prmt(wc.w, wd.w, selK0) & mskK, qb[j][0], qb[j][1]);
      }
    }

    // group-local token of accumulator row g (+1 or +8 for row g+8) in row block rb
    auto row_token = [&](int rb) { return BITS == 2 ? 16 * (g >> 2) + 4 * (g & 3) + 2 * rb : 16 * rb + rho; };
    constexpr int kRowStep = BITS == 2 ? 1 : 8;

    // ---- online softmax over the 32 tokens (exp2 domain, lazily rescaled reference)
    float pv[2][4];
    {
      float x[2][4];  // [head j][rb0 row, rb0 row+8, rb1 row, rb1 row+8]
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int rb = 0; rb < 2; ++rb) {
          x[j][2 * rb] = fmaf(s[rb][j], kmul[2 * rb], bias[j]);
          x[j][2 * rb + 1] = fmaf(s[rb][2 + j], kmul[2 * rb + 1], bias[j]);
        }
      if (tb + 32 > t_end) {  // warp-uniform: only the sequence's last group is partial
#pragma unroll
        for (int rb = 0; rb < 2; ++rb) {
          const int tr = tb + row_token(rb);
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            if (tr >= t_end) x[j][2 * rb] = -INFINITY;
            if (tr + kRowStep >= t_end) x[j][2 * rb + 1] = -INFINITY;
          }
        }
      }
      float mx[2];
      bool grow = false;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        mx[j] = fmaxf(fmaxf(x[j][0], x[j][1]), fmaxf(x[j][2], x[j][3]));
        grow |= mx[j] > mref[j];
      }
      // move the reference only when some score passed it (rare after the first tile of a
      // split): then the head maxima are reduced over the warp and alpha = 2^(old - new)
      // rescales the running sums
      if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], 4));
          mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], 8));
          mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], 16));
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float mnew = mx[j] > mref[j] ? mx[j] + kHeadroom : mref[j];
          const float alpha = mref[j] == -INFINITY ? 0.f : fast_exp2(mref[j] - mnew);
          mref[j] = mnew;
          lrow[j] *= alpha;
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            o[mt][j] *= alpha;
            o[mt][2 + j] *= alpha;
          }
          cacc[j] *= alpha;
          cacc[2 + j] *= alpha;
        }
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float muse = mref[j] == -INFINITY ? 0.f : mref[j];
        float acc = 0.f;
#pragma unroll
        for (int rb = 0; rb < 2; ++rb) {
          pv[rb][j] = fast_exp2(x[j][2 * rb] - muse);
          pv[rb][2 + j] = fast_exp2(x[j][2 * rb + 1] - muse);
          acc += pv[rb][j] + pv[rb][2 + j];
        }
        lrow[j] += acc;
      }
    }

    // ---- P' = P * s_v per group; PV and the value-minimum term on the tensor cores
    const int tw = 32 * warp;  // tile-local first token of the warp's group
    if (BITS == 2) {
      // the warp's value scales / minima as operand pairs (token, token + 4): lane = token
      const uint2 sv = *reinterpret_cast<const uint2*>(st + L::OFF_VS + (tw + lane) * 8);
      const uint2 mv = *reinterpret_cast<const uint2*>(st + L::OFF_VM + (tw + lane) * 8);
      const uint32_t svw[2] = {sv.x, sv.y}, mvw[2] = {mv.x, mv.y};
#pragma unroll
      for (int gr = 0; gr < 4; ++gr) {
        *reinterpret_cast<uint16_t*>(vp_warp + gr * 64 + vp_tok) = uint16_t(svw[gr >> 1] >> (16 * (gr & 1)));
        *reinterpret_cast<uint16_t*>(vp_warp + 256 + gr * 64 + vp_tok) = uint16_t(mvw[gr >> 1] >> (16 * (gr & 1)));
      }
      __syncwarp();
    }
#pragma unroll
    for (int rb = 0; rb < 2; ++rb) {
      uint32_t pb[4][2];
      const uint32_t hp0 = pack_f16x2(pv[rb][0], pv[rb][1]);
      const uint32_t hp1 = pack_f16x2(pv[rb][2], pv[rb][3]);
      if (BITS == 2) {
        // P transposed once into the PV B layout: k pairs (2tq, 2tq+1) / (2tq+8, 2tq+9) are the
        // tokens (T0, T0+4) / (T0+1, T0+5), T0 = 8tq + 2rb; then one scale pair per group
        const uint32_t pt0 = movmatrix_trans(hp0), pt1 = movmatrix_trans(hp1);
#pragma unroll
        for (int gr = 0; gr < 4; ++gr) {
          const uint2 sp = *reinterpret_cast<const uint2*>(vp_warp + gr * 64 + tq * 16 + rb * 8);
          pb[gr][0] = h2u(__hmul2(u2h(pt0), u2h(sp.x)));
          pb[gr][1] = h2u(__hmul2(u2h(pt1), u2h(sp.y)));
        }
        // value minima: A rows g < 4 = groups, the same token pairs
        const uint2 mp = *reinterpret_cast<const uint2*>(vp_warp + 256 + (g & 3) * 64 + tq * 16 + rb * 8);
        const uint32_t keep = g < 4 ? 0xffffffffu : 0u;
        mma_f16(cacc, mp.x & keep, 0u, mp.y & keep, 0u, pt0, pt1);
      } else {
        // value scales of the tokens of rows g and g+8 (adjacent tokens in the 2-bit form)
        const int tr = tw + row_token(rb);
        uint32_t s0w[2], s1w[2];
        if (BITS == 2) {
          const uint4 vs01 = *reinterpret_cast<const uint4*>(st + L::OFF_VS + tr * 8);
          s0w[0] = vs01.x; s0w[1] = vs01.y; s1w[0] = vs01.z; s1w[1] = vs01.w;
        } else {
          const uint2 vs0 = *reinterpret_cast<const uint2*>(st + L::OFF_VS + tr * 8);
          const uint2 vs1 = *reinterpret_cast<const uint2*>(st + L::OFF_VS + (tr + 8) * 8);
          s0w[0] = vs0.x; s0w[1] = vs0.y; s1w[0] = vs1.x; s1w[1] = vs1.y;
        }
#pragma unroll
        for (int gr = 0; gr < 4; ++gr) {
          const __half2 sa = (gr & 1) ? __high2half2(u2h(s0w[gr >> 1])) : __low2half2(u2h(s0w[gr >> 1]));
          const __half2 sb = (gr & 1) ? __high2half2(u2h(s1w[gr >> 1])) : __low2half2(u2h(s1w[gr >> 1]));
          pb[gr][0] = movmatrix_trans(h2u(__hmul2(u2h(hp0), sa)));
          pb[gr][1] = movmatrix_trans(h2u(__hmul2(u2h(hp1), sb)));
        }
      // After the transpose, MMA k index kappa (0..15) of this row block is accumulator row
      // kappa: lane tq's k pairs (2tq, 2tq+1) and (2tq+8, 2tq+9) are the tokens
      //  2-bit: tq8 + {0, 4} and tq8 + {1, 5}, tq8 = 8tq + 2rb;
      //  4-bit: tq + {0, 4} and tq + {8, 12} (+16rb).
      const int kt0 = BITS == 2 ? 8 * tq + 2 * rb : 16 * rb + tq;
      constexpr int kd1 = 4, kd2 = BITS == 2 ? 1 : 8, kd3 = BITS == 2 ? 5 : 12;
      {
        // value minima: A rows = groups (rows g < 4)
        const uint32_t pt0 = movmatrix_trans(hp0), pt1 = movmatrix_trans(hp1);
        const uint8_t* vmr = st + L::OFF_VM + 2 * (g & 3) + (tw + kt0) * 8;
        const uint32_t keep = g < 4 ? 0xffffffffu : 0u;
        const uint32_t a0 = (lds_u16(vmr) | (lds_u16(vmr + kd1 * 8) << 16)) & keep;
        const uint32_t a2 = (lds_u16(vmr + kd2 * 8) | (lds_u16(vmr + kd3 * 8) << 16)) & keep;
        mma_f16(cacc, a0, 0u, a2, 0u, pt0, pt1);
      }
      }
      if (BITS == 2) {
        // tokens tw + kt0 + {0, 4, 1, 5} sit at interleaved rows (kt0 + d) * 16 + tq + 4 warp
        const uint8_t* vt = st + L::OFF_VQ + v_lane + (2 * rb) * 512;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          // word 2i + (g >> 2) (byte offset 8i + 4(g >> 2), the latter in v_lane)
          const uint32_t rA = prmt(lds_u32(vt + 8 * i), lds_u32(vt + 4 * 512 + 8 * i), selV0);
          const uint32_t rC = prmt(lds_u32(vt + 1 * 512 + 8 * i), lds_u32(vt + 5 * 512 + 8 * i), selV0);
          mma_f16(o[2 * i], rA & 0x00030003u, rA & 0x000C000Cu, rC & 0x00030003u, rC & 0x000C000Cu, pb[i][0],
                  pb[i][1]);
          mma_f16(o[2 * i + 1], rA & 0x00300030u, rA & 0x00C000C0u, rC & 0x00300030u, rC & 0x00C000C0u, pb[i][0],
                  pb[i][1]);
        }
      } else {
        const int tl = tw + 16 * rb;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t W[4][8];  // [u][word]: word i holds channels 64*half + 8i .. +7
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint8_t* row = st + L::OFF_VQ + (tl + tq + 4 * u) * L::VQ_PITCH + half * 32;
            const uint4 lo = *reinterpret_cast<const uint4*>(row);
            const uint4 hi = *reinterpret_cast<const uint4*>(row + 16);
            W[u][0] = lo.x; W[u][1] = lo.y; W[u][2] = lo.z; W[u][3] = lo.w;
            W[u][4] = hi.x; W[u][5] = hi.y; W[u][6] = hi.z; W[u][7] = hi.w;
          }
#pragma unroll
          for (int ml = 0; ml < 4; ++ml) {
            const int mt = 4 * half + ml;
            mma_f16(o[mt], prmt(W[0][2 * ml], W[1][2 * ml], selV0) & mskV,
                    prmt(W[0][2 * ml + 1], W[1][2 * ml + 1], selV0) & mskV,
                    prmt(W[2][2 * ml], W[3][2 * ml], selV0) & mskV,
                    prmt(W[2][2 * ml + 1], W[3][2 * ml + 1], selV0) & mskV, pb[mt >> 1][0], pb[mt >> 1][1]);
          }
        }
      }
    }
  }

  // ---- epilogue: reduce over rows, merge warps, write split partials
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    float l = lrow[j];
    l += __shfl_xor_sync(0xffffffffu, l, 4);
    l += __shfl_xor_sync(0xffffffffu, l, 8);
    l += __shfl_xor_sync(0xffffffffu, l, 16);
    lrow[j] = l;
  }
  // value-minimum term of group gr for heads 2tq+j lives in lane (gr, tq)
  float corr[4][2];
#pragma unroll
  for (int gr = 0; gr < 4; ++gr) {
    corr[gr][0] = __shfl_sync(0xffffffffu, cacc[0], gr * 4 + tq);
    corr[gr][1] = __shfl_sync(0xffffffffu, cacc[1], gr * 4 + tq);
  }
  cp_async_wait<0>();
  __syncthreads();
  float* red_m = reinterpret_cast<float*>(smem);  // [4][8]
  float* red_l = red_m + kWarpsK * 8;             // [4][8]
  float* red_o = red_l + kWarpsK * 8;             // [4][8][kRedPitch]
  if (g == 0) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      red_m[warp * 8 + 2 * tq + j] = mref[j];
      red_l[warp * 8 + 2 * tq + j] = lrow[j];
    }
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int h = 2 * tq + j;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarpsK; ++w) M = fmaxf(M, red_m[w * 8 + h]);
    const float f = (M == -INFINITY) ? 0.f : fast_exp2(mref[j] - M);
    float* ro = red_o + (warp * 8 + h) * kRedPitch;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      if (BITS == 2) {
        // rows g / g+8 of m-tile mt: adjacent channels ca, ca+1, field positions 2(mt&1) + {0, 1}
        const int ca = 16 * (2 * (mt >> 1) + (g >> 2)) + 4 * (g & 3) + 2 * (mt & 1);
        const float sv0 = __int_as_float((127 + 24 - 4 * (mt & 1)) << 23);
        const float sv1 = __int_as_float((127 + 22 - 4 * (mt & 1)) << 23);
        *reinterpret_cast<float2*>(ro + ca) = make_float2(fmaf(o[mt][j], sv0, corr[mt >> 1][j]) * f,
                                                          fmaf(o[mt][2 + j], sv1, corr[mt >> 1][j]) * f);
      } else {
        const int ca = 16 * mt + g;  // A row g; row g+8 is channel ca + 8
        ro[ca] = fmaf(o[mt][j], subV, corr[mt >> 1][j]) * f;
        ro[ca + 8] = fmaf(o[mt][2 + j], subV, corr[mt >> 1][j]) * f;
      }
    }
  }
  __syncthreads();
  // thread = channel; heads in turn. The (max, sum) of each head comes from its channel-0 thread.
  const int c = threadIdx.x;
  const int64_t pi0 = (int64_t(b) * p.Hq + hk * p.G + h0) * p.split_stride + split;
  for (int h = 0; h < nheads; ++h) {
    float O = 0.f;
#pragma unroll
    for (int w = 0; w < kWarpsK; ++w) O += red_o[(w * 8 + h) * kRedPitch + c];
    const int64_t pi = pi0 + int64_t(h) * p.split_stride;
    p.part_o[pi * 128 + c] = O;
    if (c == 0) {
      float M = -INFINITY, Lsum = 0.f;
#pragma unroll
      for (int w = 0; w < kWarpsK; ++w) M = fmaxf(M, red_m[w * 8 + h]);
#pragma unroll
      for (int w = 0; w < kWarpsK; ++w)
        Lsum += (M == -INFINITY) ? 0.f : red_l[w * 8 + h] * fast_exp2(red_m[w * 8 + h] - M);
      p.part_m[pi] = M * kLn2K;
      p.part_l[pi] = Lsum;
    }
  }
}

// ---- TMA tensor maps (host). Encoded through the driver entry point fetched from the
// runtime (no link against libcuda) and cached per cache-tensor geometry, so a decode loop
// over the same caches encodes once.
struct TmaKey {
  const void* kq; const void* vq; const void* vs; const void* vm;
  int64_t W, Sq, Hk, B, kq_sc, kq_sh, kq_sb, vq_st, vq_sh, vq_sb, vs_sh, vs_sb, vm_sh, vm_sb;
  int dev;
};
struct TmaEntry {
  TmaKey key;
  CUtensorMap m[4];
  bool used;
};
std::mutex g_tma_mu;
TmaEntry g_tma[16];
int g_tma_next = 0;

// The 2-bit TMA form needs 16-byte aligned bases and strides (bytes), dense 32-byte value
// rows (the value map splits the token index into token / 8 and token % 8, so the box lands
// in the interleaved row order of the value tile) and dense 8-byte rows of value
// scales/minima (read as 16-byte rows of two tokens). W = words per key row.
bool kivi_tma_maps(const KiviParams& kp, int64_t W, CUtensorMap out[4]) {
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  // bytes stride of a dim, or a harmless 16-byte multiple when the dim has one entry
  auto st = [](int64_t elems, int esz, int64_t size, int64_t fallback) -> int64_t {
    return size > 1 ? elems * esz : fallback;
  };
  const int64_t Hk = kp.Hk, B = kp.B, Sq = kp.Sq;
  const int64_t s_kc = kp.kq_sc * 4, s_kh = st(kp.kq_sh, 4, Hk, s_kc * 128), s_kb = st(kp.kq_sb, 4, B, s_kh * Hk);
  const int64_t s_vt = kp.vq_st * 4, s_vh = st(kp.vq_sh, 4, Hk, s_vt * Sq), s_vb = st(kp.vq_sb, 4, B, s_vh * Hk);
  const int64_t s_sh = st(kp.vs_sh, 2, Hk, Sq * 8), s_sb = st(kp.vs_sb, 2, B, s_sh * Hk);
  const int64_t s_mh = st(kp.vm_sh, 2, Hk, Sq * 8), s_mb = st(kp.vm_sb, 2, B, s_mh * Hk);
  for (int64_t x : {s_kc, s_kh, s_kb, s_vt, s_vh, s_vb, s_sh, s_sb, s_mh, s_mb})
    if (x <= 0 || x % 16 || x >= (int64_t(1) << 40)) return false;
  if (!a16(kp.kq) || !a16(kp.vq) || !a16(kp.vs) || !a16(kp.vm) || kp.vs_st != 4 || kp.vm_st != 4 || kp.vq_st != 8 ||
      (Sq & 7))
    return false;
  TmaKey key{};
  key.kq = kp.kq; key.vq = kp.vq; key.vs = kp.vs; key.vm = kp.vm;
  key.W = W; key.Sq = Sq; key.Hk = Hk; key.B = B;
  key.kq_sc = s_kc; key.kq_sh = s_kh; key.kq_sb = s_kb; key.vq_st = s_vt; key.vq_sh = s_vh; key.vq_sb = s_vb;
  key.vs_sh = s_sh; key.vs_sb = s_sb; key.vm_sh = s_mh; key.vm_sb = s_mb;
  cudaGetDevice(&key.dev);
  std::lock_guard<std::mutex> lock(g_tma_mu);
  for (const TmaEntry& e : g_tma)
    if (e.used && std::memcmp(&e.key, &key, sizeof key) == 0) {
      std::memcpy(out, e.m, sizeof e.m);
      return true;
    }
  CUtensorMap m[4];
  const cuuint64_t dk[4] = {cuuint64_t(W), 128, cuuint64_t(Hk), cuuint64_t(B)};
  const cuuint64_t sk[3] = {cuuint64_t(s_kc), cuuint64_t(s_kh), cuuint64_t(s_kb)};
  const cuuint32_t bk[4] = {8, 128, 1, 1};
  const cuuint64_t dv[5] = {8, cuuint64_t(Sq / 8), 8, cuuint64_t(Hk), cuuint64_t(B)};
  const cuuint64_t sv[4] = {cuuint64_t(8 * s_vt), cuuint64_t(s_vt), cuuint64_t(s_vh), cuuint64_t(s_vb)};
  const cuuint32_t bv[5] = {8, uint32_t(kTile / 8), 8, 1, 1};
  const cuuint64_t ds[4] = {8, cuuint64_t(Sq / 2), cuuint64_t(Hk), cuuint64_t(B)};
  const cuuint64_t ss[3] = {16, cuuint64_t(s_sh), cuuint64_t(s_sb)};
  const cuuint64_t sm[3] = {16, cuuint64_t(s_mh), cuuint64_t(s_mb)};
  const cuuint32_t bs[4] = {8, uint32_t(kTile / 2), 1, 1};
  if (!encode_map(&m[0], CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, kp.kq, dk, sk, bk, CU_TENSOR_MAP_SWIZZLE_32B) ||
      !encode_map(&m[1], CU_TENSOR_MAP_DATA_TYPE_UINT32, 5, kp.vq, dv, sv, bv, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode_map(&m[2], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, kp.vs, ds, ss, bs, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode_map(&m[3], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, kp.vm, ds, sm, bs, CU_TENSOR_MAP_SWIZZLE_NONE))
    return false;
  TmaEntry& e = g_tma[g_tma_next];
  g_tma_next = (g_tma_next + 1) % 16;
  e.key = key;
  std::memcpy(e.m, m, sizeof m);
  e.used = true;
  std::memcpy(out, m, sizeof m);
  return true;
}

template <int BITS, bool TMA, int MINB>
int launch_kivi_as(const KiviParams& kp, int n_splits, const CUtensorMap* maps, cudaStream_t st) {
  using L = KL<BITS, TMA>;
  const size_t smem = std::max<size_t>(L::SMEM, (2 * 4 * 8 + 4 * 8 * kRedPitch) * sizeof(float)) + (TMA ? 1024 : 0);
  auto kern = kivi_decode_kernel<BITS, TMA, MINB>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    int rc = cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
                        "cudaFuncSetAttribute(kivi)");
    if (rc) return rc;
    attr[dev & 63] = true;
  }
  dim3 grid(n_splits, kp.Hk * kp.head_chunks, kp.B);
  kern<<<grid, kWarpsK * 32, smem, st>>>(kp, maps[0], maps[1], maps[2], maps[3]);
  return cuda_check(cudaGetLastError(), "kivi_decode_kernel launch");
}

// W = words per key row (Kq's last dim). 2-bit caches whose geometry TMA can address take
// the TMA form; everything else the cp.async form.
template <int BITS>
int launch_kivi(const KiviParams& kp, int n_splits, int64_t W, int ctas_per_sm, cudaStream_t st) {
  alignas(64) CUtensorMap maps[4];
  std::memset(maps, 0, sizeof maps);
  const bool four = ctas_per_sm == 4;
  if (BITS == 2 && kivi_tma_maps(kp, W, maps))
    return four ? launch_kivi_as<2, true, 4>(kp, n_splits, maps, st) : launch_kivi_as<2, true, 3>(kp, n_splits, maps, st);
  return four ? launch_kivi_as<BITS, false, 4>(kp, n_splits, maps, st)
              : launch_kivi_as<BITS, false, 3>(kp, n_splits, maps, st);
}

struct KiviPlan {
  int n_kivi, ntiles, n_res, head_chunks;
  int ctas_per_sm;  // occupancy the split count is balanced for (and the kernel compiled for)
};

int kivi_plan(int64_t B, int64_t Hq, int64_t Hk, int64_t Sq, int64_t R, KiviPlan* pl) {
  const int G = int(Hq / Hk);
  pl->head_chunks = (G + 7) / 8;
  const int64_t ntiles = (Sq + kTile - 1) / kTile;
  const int64_t pairs = B * Hk * pl->head_chunks;
  // three CTAs per SM while each split streams few tiles: the room left over lets the
  // residual-window CTAs, launched behind this pass, run beside it, which shortens the
  // step's tail; four when the packed pass is long and its own throughput dominates
  // (measured step: 16K 31.1 us at three against 32.1 at four; 32K 48.5 at three against
  // 47.1 at four)
  pl->ctas_per_sm = ntiles > 128 ? 4 : 3;
  const int64_t slots = int64_t(pl->ctas_per_sm) * num_sms();
  int64_t splits = pairs >= slots ? 1 : slots / std::max<int64_t>(pairs, 1);
  splits = std::max<int64_t>(1, std::min<int64_t>(splits, std::max<int64_t>(ntiles, 1)));
  pl->n_kivi = ntiles > 0 ? int(splits) : 0;
  pl->ntiles = int(ntiles);
  pl->n_res = R > 0 ? std::max(1, dense_split_count(B, Hq, Hk, R, 128, int(pairs))) : 0;
  return BD_OK;
}

int check_kivi_inputs(const bd_tensor* Q, const bd_tensor* Kq, const bd_tensor* Ks, const bd_tensor* Km,
                      const bd_tensor* Kr, const bd_tensor* Vq, const bd_tensor* Vs, const bd_tensor* Vm,
                      const bd_tensor* Vr, int bits, int group_size) {
  int rc;
  if (bits != 2 && bits != 4) return fail(BD_ERR_VALUE, "bits must be 2 or 4");
  if (group_size != 32) return fail(BD_ERR_UNSUPPORTED, "group_size must be 32");
  if ((rc = check_tensor(Q, "Q", 3)) || (rc = check_tensor(Kq, "Kq", 4, BD_I32)) ||
      (rc = check_tensor(Ks, "K_scale", 4, BD_F16)) || (rc = check_tensor(Km, "K_mn", 4, BD_F16)) ||
      (rc = check_tensor(Kr, "K_residual", 4, BD_BF16)) || (rc = check_tensor(Vq, "Vq", 4, BD_I32)) ||
      (rc = check_tensor(Vs, "V_scale", 4, BD_F16)) || (rc = check_tensor(Vm, "V_mn", 4, BD_F16)) ||
      (rc = check_tensor(Vr, "V_residual", 4, BD_BF16)))
    return rc;
  if (Q->dtype != BD_BF16 && Q->dtype != BD_F16 && Q->dtype != BD_F32)
    return fail(BD_ERR_DTYPE, "Q must be bf16, f16 or f32");
  const int64_t B = Q->shape[0], Hq = Q->shape[1], D = Q->shape[2];
  const int64_t Hk = Kq->shape[1];
  const int fpi = 32 / bits;
  if (D != 128) return fail(BD_ERR_UNSUPPORTED, "KIVI decode supports head_dim 128");
  if (Hk <= 0 || Hq % Hk) return fail(BD_ERR_SHAPE, "H_q must be a multiple of H_k");
  const int64_t Sq = Kq->shape[3] * fpi;
  if (Kq->shape[0] != B || Kq->shape[2] != D) return fail(BD_ERR_SHAPE, "Kq must be [B,Hk,D,Sq/fpi]");
  for (const bd_tensor* t : {Ks, Km})
    if (t->shape[0] != B || t->shape[1] != Hk || t->shape[2] != D || t->shape[3] * 32 != Sq)
      return fail(BD_ERR_SHAPE, "K_scale/K_mn must be [B,Hk,D,Sq/32]");
  if (Vq->shape[0] != B || Vq->shape[1] != Hk || Vq->shape[2] != Sq || Vq->shape[3] * fpi != D)
    return fail(BD_ERR_SHAPE, "Vq must be [B,Hk,Sq,D/fpi], Sq matching Kq");
  for (const bd_tensor* t : {Vs, Vm})
    if (t->shape[0] != B || t->shape[1] != Hk || t->shape[2] != Sq || t->shape[3] * 32 != D)
      return fail(BD_ERR_SHAPE, "V_scale/V_mn must be [B,Hk,Sq,D/32]");
  for (const bd_tensor* t : {Kr, Vr})
    if (t->shape[0] != B || t->shape[1] != Hk || t->shape[3] != D || t->shape[2] != Kr->shape[2])
      return fail(BD_ERR_SHAPE, "K_residual/V_residual must be [B,Hk,R,D]");
  if ((rc = check_rows_aligned(Kq, "Kq", 16)) || (rc = check_rows_aligned(Vq, "Vq", 16)) ||
      (rc = check_rows_aligned(Ks, "K_scale", 8)) || (rc = check_rows_aligned(Km, "K_mn", 8)) ||
      (rc = check_rows_aligned(Vs, "V_scale", 8)) || (rc = check_rows_aligned(Vm, "V_mn", 8)))
    return rc;
  if (Q->stride[2] != 1) return fail(BD_ERR_STRIDE, "Q innermost dim must be contiguous");
  return BD_OK;
}

__global__ void empty_partials_kernel(float* m, float* l, float* o, int rows, int D) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  m[r] = -INFINITY;
  l[r] = 0.f;
  for (int c = 0; c < D; ++c) o[int64_t(r) * D + c] = 0.f;
}

// ---------------------------------------------------------------- KIVI pack
template <typename T, int BITS>
__global__ void kivi_pack_kernel(const T* __restrict__ x, int nlead, int64_t l0, int64_t l1, int64_t l2,
                                 int64_t s0, int64_t s1, int64_t s2, int N, int64_t total_groups,
                                 uint32_t* __restrict__ code, T* __restrict__ scale, T* __restrict__ mn) {
  const int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= total_groups) return;
  const int gpr = N / 32;
  const int64_t row = gid / gpr;
  const int grp = int(gid % gpr);
  // row -> (i0, i1, i2) over up to three leading dims
  const int64_t i2 = row % l2, r1 = row / l2;
  const int64_t i1 = r1 % l1, i0 = r1 / l1;
  const T* src = x + i0 * s0 + i1 * s1 + i2 * s2 + int64_t(grp) * 32;
  float v[32];
#pragma unroll
  for (int e = 0; e < 32; ++e) v[e] = to_f32<T>(src[e]);
  float lo = v[0], hi = v[0];
#pragma unroll
  for (int e = 1; e < 32; ++e) { lo = fminf(lo, v[e]); hi = fmaxf(hi, v[e]); }
  constexpr int LV = (1 << BITS) - 1;
  // (max-min)/(2^bits-1) as PyTorch forms it on a CUDA device: times the fp32 reciprocal
  constexpr float kRcp = 1.0f / float(LV);
  const float sc = __fmul_rn(fmaxf(__fsub_rn(hi, lo), 1e-8f), kRcp);
  constexpr int FPI = 32 / BITS;
  uint32_t words[32 / FPI];
#pragma unroll
  for (int w = 0; w < 32 / FPI; ++w) words[w] = 0u;
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    float qv = rintf(__fdiv_rn(__fsub_rn(v[e], lo), sc));
    qv = fminf(fmaxf(qv, 0.f), float(LV));
    words[e / FPI] |= uint32_t(qv) << ((e % FPI) * BITS);
  }
  const int64_t wbase = row * (N / FPI) + int64_t(grp) * (32 / FPI);
#pragma unroll
  for (int w = 0; w < 32 / FPI; ++w) code[wbase + w] = words[w];
  scale[row * gpr + grp] = from_f32<T>(sc);
  mn[row * gpr + grp] = from_f32<T>(lo);
}

// ---------------------------------------------------------------- KIVI cache append
// Quantizes whole 32-token groups of new keys/values into existing packed caches at a
// token offset, with the packer's arithmetic (fp32 min/max, scale = max(max-min,1e-8) times
// the fp32 reciprocal of 2^bits-1, round-half-even, clamp): the caches then hold exactly what packing the whole
// sequence at once would give. Keys are quantized per channel over the group's tokens
// (one thread per (b, hk, channel, group); a warp reads 32 consecutive channels of each
// token), values per token over 32-channel groups (one thread per (b, hk, token, group)).
struct AppendParams {
  const void* k; int64_t k_sb, k_sh, k_st;  // [B,Hk,Tn,D], channels contiguous
  const void* v; int64_t v_sb, v_sh, v_st;
  int in_dtype;
  int B, Hk, Tn, D;
  int64_t t0;  // token offset of the first new token (multiple of 32)
  uint32_t* kq; int64_t kq_sb, kq_sh, kq_sc;  // [B,Hk,D,cap/fpi]
  __half* ks; int64_t ks_sb, ks_sh, ks_sc;    // [B,Hk,D,cap/32]
  __half* km; int64_t km_sb, km_sh, km_sc;
  uint32_t* vq; int64_t vq_sb, vq_sh, vq_st;  // [B,Hk,cap,D/fpi]
  __half* vs; int64_t vs_sb, vs_sh, vs_st;    // [B,Hk,cap,D/32]
  __half* vm; int64_t vm_sb, vm_sh, vm_st;
};

__device__ __forceinline__ float ld_in(const void* base, int dt, int64_t off) {
  switch (dt) {
    case BD_F16: return __half2float(reinterpret_cast<const __half*>(base)[off]);
    case BD_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[off]);
    default: return reinterpret_cast<const float*>(base)[off];
  }
}

// quantize 32 values, return the packed words, scale and minimum
template <int BITS>
__device__ __forceinline__ void quant32(const float* v, uint32_t* words, float* sc_out, float* lo_out) {
  float lo = v[0], hi = v[0];
#pragma unroll
  for (int e = 1; e < 32; ++e) { lo = fminf(lo, v[e]); hi = fmaxf(hi, v[e]); }
  constexpr int LV = (1 << BITS) - 1;
  constexpr int FPI = 32 / BITS;
  constexpr float kRcp = 1.0f / float(LV);
  const float sc = __fmul_rn(fmaxf(__fsub_rn(hi, lo), 1e-8f), kRcp);
#pragma unroll
  for (int w = 0; w < 32 / FPI; ++w) words[w] = 0u;
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    float qv = rintf(__fdiv_rn(__fsub_rn(v[e], lo), sc));
    qv = fminf(fmaxf(qv, 0.f), float(LV));
    words[e / FPI] |= uint32_t(qv) << ((e % FPI) * BITS);
  }
  *sc_out = sc;
  *lo_out = lo;
}

template <int BITS>
__global__ void kivi_append_kernel(const AppendParams p) {
  constexpr int FPI = 32 / BITS;
  const int ngr = p.Tn / 32;
  const int64_t nk = int64_t(p.B) * p.Hk * ngr * p.D;  // key threads: (b, hk, group, channel)
  const int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  float v[32];
  uint32_t words[32 / FPI];
  float sc, lo;
  if (gid < nk) {
    const int c = int(gid % p.D);
    int64_t r = gid / p.D;
    const int grp = int(r % ngr); r /= ngr;
    const int hk = int(r % p.Hk), b = int(r / p.Hk);
    const int64_t base = int64_t(b) * p.k_sb + int64_t(hk) * p.k_sh + int64_t(grp) * 32 * p.k_st + c;
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = ld_in(p.k, p.in_dtype, base + int64_t(e) * p.k_st);
    quant32<BITS>(v, words, &sc, &lo);
    const int64_t g0 = p.t0 / 32 + grp;  // group index in the cache
    uint32_t* kq = p.kq + int64_t(b) * p.kq_sb + int64_t(hk) * p.kq_sh + int64_t(c) * p.kq_sc + g0 * (32 / FPI);
#pragma unroll
    for (int w = 0; w < 32 / FPI; ++w) kq[w] = words[w];
    p.ks[int64_t(b) * p.ks_sb + int64_t(hk) * p.ks_sh + int64_t(c) * p.ks_sc + g0] = __float2half_rn(sc);
    p.km[int64_t(b) * p.km_sb + int64_t(hk) * p.km_sh + int64_t(c) * p.km_sc + g0] = __float2half_rn(lo);
    return;
  }
  const int64_t vid = gid - nk;  // value threads: (b, hk, token, channel group)
  const int cg = p.D / 32;
  if (vid >= int64_t(p.B) * p.Hk * p.Tn * cg) return;
  const int grp = int(vid % cg);
  int64_t r = vid / cg;
  const int t = int(r % p.Tn); r /= p.Tn;
  const int hk = int(r % p.Hk), b = int(r / p.Hk);
  const int64_t base = int64_t(b) * p.v_sb + int64_t(hk) * p.v_sh + int64_t(t) * p.v_st + grp * 32;
#pragma unroll
  for (int e = 0; e < 32; ++e) v[e] = ld_in(p.v, p.in_dtype, base + e);
  quant32<BITS>(v, words, &sc, &lo);
  const int64_t tc = p.t0 + t;  // token index in the cache
  uint32_t* vq = p.vq + int64_t(b) * p.vq_sb + int64_t(hk) * p.vq_sh + tc * p.vq_st + grp * (32 / FPI);
#pragma unroll
  for (int w = 0; w < 32 / FPI; ++w) vq[w] = words[w];
  p.vs[int64_t(b) * p.vs_sb + int64_t(hk) * p.vs_sh + tc * p.vs_st + grp] = __float2half_rn(sc);
  p.vm[int64_t(b) * p.vm_sb + int64_t(hk) * p.vm_sh + tc * p.vm_st + grp] = __float2half_rn(lo);
}

// ---------------------------------------------------------------- KIVI GEMV
// out[b,hq,m,n] = sum_k fA[b,hq,m,k] * (code(qB[b,hk,k,n]) * sc[b,hk,k,n/gs] + zr[b,hk,k,n/gs])
struct GemvParams {
  const __half* fa; int64_t fa_sb, fa_sh, fa_sm;
  const uint32_t* qb; int64_t qb_sb, qb_sh, qb_sk;
  const __half* sc; int64_t sc_sb, sc_sh, sc_sk;
  const __half* zr; int64_t zr_sb, zr_sh, zr_sk;
  __half* out; int64_t o_sb, o_sh, o_sm;
  int B, Hq, Hk, M, K, N, bits, gs;
};

__global__ void kivi_gemv_kernel(const GemvParams p) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / p.Hq, hq = bh % p.Hq, hk = hq / (p.Hq / p.Hk);
  if (n >= p.N) return;
  const int fpi = 32 / p.bits;
  const uint32_t mask = (1u << p.bits) - 1u;
  const int sh = (n % fpi) * p.bits;
  const uint32_t* qrow = p.qb + int64_t(b) * p.qb_sb + int64_t(hk) * p.qb_sh + n / fpi;
  const __half* srow = p.sc + int64_t(b) * p.sc_sb + int64_t(hk) * p.sc_sh + n / p.gs;
  const __half* zrow = p.zr + int64_t(b) * p.zr_sb + int64_t(hk) * p.zr_sh + n / p.gs;
  for (int m = 0; m < p.M; ++m) {
    const __half* arow = p.fa + int64_t(b) * p.fa_sb + int64_t(hq) * p.fa_sh + int64_t(m) * p.fa_sm;
    float acc = 0.f;
    for (int k = 0; k < p.K; ++k) {
      const float c = float((qrow[int64_t(k) * p.qb_sk] >> sh) & mask);
      const float w = c * __half2float(srow[int64_t(k) * p.sc_sk]) + __half2float(zrow[int64_t(k) * p.zr_sk]);
      acc = fmaf(__half2float(arow[k]), w, acc);
    }
    p.out[int64_t(b) * p.o_sb + int64_t(hq) * p.o_sh + int64_t(m) * p.o_sm + n] = __float2half_rn(acc);
  }
}

}  // namespace
}  // namespace bd

namespace bd {
// host read of this file's wait-timeout counter (-1 on failure)
long long kivi_wait_timeouts() {
  unsigned int v = 0;
  return cudaMemcpyFromSymbol(&v, g_kivi_tma_timeouts, sizeof v) == cudaSuccess ? (long long)v : -1;
}
}  // namespace bd

extern "C" {

size_t bd_kivi_decode_attn_workspace(const bd_tensor* Q, const bd_tensor* Kq, const bd_tensor* K_residual,
                                     int bits) {
  using namespace bd;
  if (check_tensor(Q, "Q", 3) || check_tensor(Kq, "Kq", 4) || check_tensor(K_residual, "K_residual", 4)) return 0;
  if (bits != 2 && bits != 4) return 0;
  KiviPlan pl;
  kivi_plan(Q->shape[0], Q->shape[1], Kq->shape[1], Kq->shape[3] * (32 / bits), K_residual->shape[2], &pl);
  return partials_bytes(size_t(Q->shape[0] * Q->shape[1]), std::max(1, pl.n_kivi + pl.n_res), 128);
}

int bd_kivi_decode_attn_stages(const bd_tensor* Q, const bd_tensor* Kq, const bd_tensor* K_scale,
                               const bd_tensor* K_mn, const bd_tensor* K_residual, const bd_tensor* Vq,
                               const bd_tensor* V_scale, const bd_tensor* V_mn, const bd_tensor* V_residual, int bits,
                               int group_size, float scaling, const bd_tensor* out, void* workspace,
                               size_t workspace_bytes, int stages, bd_stream_t stream);

int bd_kivi_decode_attn(const bd_tensor* Q, const bd_tensor* Kq, const bd_tensor* K_scale, const bd_tensor* K_mn,
                        const bd_tensor* K_residual, const bd_tensor* Vq, const bd_tensor* V_scale,
                        const bd_tensor* V_mn, const bd_tensor* V_residual, int bits, int group_size, float scaling,
                        const bd_tensor* out, void* workspace, size_t workspace_bytes, bd_stream_t stream) {
  return bd_kivi_decode_attn_stages(Q, Kq, K_scale, K_mn, K_residual, Vq, V_scale, V_mn, V_residual, bits, group_size,
                                    scaling, out, workspace, workspace_bytes, 7, stream);
}

int bd_kivi_decode_attn_stages(const bd_tensor* Q, const bd_tensor* Kq, const bd_tensor* K_scale,
                               const bd_tensor* K_mn, const bd_tensor* K_residual, const bd_tensor* Vq,
                               const bd_tensor* V_scale, const bd_tensor* V_mn, const bd_tensor* V_residual, int bits,
                               int group_size, float scaling, const bd_tensor* out, void* workspace,
                               size_t workspace_bytes, int stages, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if ((rc = check_kivi_inputs(Q, Kq, K_scale, K_mn, K_residual, Vq, V_scale, V_mn, V_residual, bits, group_size)))
    return rc;
  if ((rc = check_tensor(out, "out", 3))) return rc;
  if (out->dtype != BD_BF16 && out->dtype != BD_F16 && out->dtype != BD_F32)
    return fail(BD_ERR_DTYPE, "out must be bf16, f16 or f32");
  for (int i = 0; i < 3; ++i)
    if (out->shape[i] != Q->shape[i]) return fail(BD_ERR_SHAPE, "out must have Q's shape");
  if (out->stride[2] != 1) return fail(BD_ERR_STRIDE, "out innermost dim must be contiguous");
  const int64_t B = Q->shape[0], Hq = Q->shape[1], Hk = Kq->shape[1];
  const int64_t Sq = Kq->shape[3] * (32 / bits), R = K_residual->shape[2];
  if (B * Hq == 0) return BD_OK;
  KiviPlan pl;
  kivi_plan(B, Hq, Hk, Sq, R, &pl);
  const int ntot = std::max(1, pl.n_kivi + pl.n_res);
  const size_t need = partials_bytes(size_t(B * Hq), ntot, 128);
  if (!workspace || workspace_bytes < need)
    return fail(BD_ERR_WORKSPACE, "need " + std::to_string(need) + " workspace bytes");
  Partials part = carve_partials(workspace, size_t(B * Hq), ntot, 128);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (pl.n_kivi + pl.n_res == 0) {
    // no keys at all: one empty partial per row -> NaN output like the reference's 0/0
    const int rows = int(B * Hq);
    empty_partials_kernel<<<(rows + 127) / 128, 128, 0, st>>>(part.m, part.l, part.o, rows, 128);
    if ((rc = cuda_check(cudaGetLastError(), "empty_partials_kernel launch"))) return rc;
    return launch_combine(part, int(B), int(Hq), 128, out, st);
  }
  if (pl.n_kivi > 0 && (stages & 1)) {
    KiviParams kp{};
    kp.q = Q->data; kp.q_sb = Q->stride[0]; kp.q_sh = Q->stride[1]; kp.q_dtype = Q->dtype;
    kp.kq = static_cast<const uint32_t*>(Kq->data); kp.kq_sb = Kq->stride[0]; kp.kq_sh = Kq->stride[1]; kp.kq_sc = Kq->stride[2];
    kp.ks = static_cast<const __half*>(K_scale->data); kp.ks_sb = K_scale->stride[0]; kp.ks_sh = K_scale->stride[1]; kp.ks_sc = K_scale->stride[2];
    kp.km = static_cast<const __half*>(K_mn->data); kp.km_sb = K_mn->stride[0]; kp.km_sh = K_mn->stride[1]; kp.km_sc = K_mn->stride[2];
    kp.vq = static_cast<const uint32_t*>(Vq->data); kp.vq_sb = Vq->stride[0]; kp.vq_sh = Vq->stride[1]; kp.vq_st = Vq->stride[2];
    kp.vs = static_cast<const __half*>(V_scale->data); kp.vs_sb = V_scale->stride[0]; kp.vs_sh = V_scale->stride[1]; kp.vs_st = V_scale->stride[2];
    kp.vm = static_cast<const __half*>(V_mn->data); kp.vm_sb = V_mn->stride[0]; kp.vm_sh = V_mn->stride[1]; kp.vm_st = V_mn->stride[2];
    kp.B = int(B); kp.Hq = int(Hq); kp.Hk = int(Hk); kp.G = int(Hq / Hk); kp.Sq = int(Sq);
    kp.head_chunks = pl.head_chunks; kp.nsplit = pl.n_kivi; kp.ntiles = pl.ntiles;
    kp.scale_log2 = scaling * kLog2eK;
    kp.part_m = part.m; kp.part_l = part.l; kp.part_o = part.o; kp.split_stride = ntot;
    rc = bits == 2 ? launch_kivi<2>(kp, pl.n_kivi, Kq->shape[3], pl.ctas_per_sm, st)
                   : launch_kivi<4>(kp, pl.n_kivi, Kq->shape[3], pl.ctas_per_sm, st);
    if (rc) return rc;
  }
  if (pl.n_res == 1 && pl.n_kivi > 0 && (stages & 7) == 7) {
    // one window CTA per group: it waits for the packed pass and merges the group's split
    // slots itself, so no combine kernel runs
    return launch_dense_merge(Q, K_residual, V_residual, scaling, part, pl.n_kivi, out, st);
  }
  if (pl.n_res > 0 && (stages & 2)) {
    // programmatic dependent of the KIVI pass when that ran just before it
    const bool pdl = pl.n_kivi > 0 && (stages & 1);
    if ((rc = launch_dense_partials(Q, K_residual, V_residual, scaling, part, pl.n_kivi, pl.n_res, st, pdl)))
      return rc;
  }
  if (!(stages & 4)) return BD_OK;
  return launch_combine(part, int(B), int(Hq), 128, out, st, (stages & 3) != 0);
}

int bd_kivi_pack_last_dim(const bd_tensor* x, int group_size, int bits, const bd_tensor* code,
                          const bd_tensor* scale, const bd_tensor* mn, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if (!x) return fail(BD_ERR_NULL, "x is NULL");
  if (bits != 2 && bits != 4 && bits != 8) return fail(BD_ERR_VALUE, "bits must be 2, 4 or 8");
  if (group_size != 32) return fail(BD_ERR_UNSUPPORTED, "group_size must be 32");
  const int nd = x->ndim;
  if (nd < 1 || nd > 4) return fail(BD_ERR_SHAPE, "x must have 1 to 4 dims");
  if ((rc = check_tensor(x, "x", nd)) || (rc = check_tensor(code, "code", nd, BD_I32)) ||
      (rc = check_tensor(scale, "scale", nd, x->dtype)) || (rc = check_tensor(mn, "mn", nd, x->dtype)))
    return rc;
  if (x->dtype != BD_F16 && x->dtype != BD_BF16 && x->dtype != BD_F32)
    return fail(BD_ERR_DTYPE, "x must be f16, bf16 or f32");
  const int64_t N = x->shape[nd - 1];
  if (N % 32) return fail(BD_ERR_SHAPE, "last dim must be a multiple of 32");
  if (x->stride[nd - 1] != 1 && N > 1) return fail(BD_ERR_STRIDE, "x innermost dim must be contiguous");
  const int fpi = 32 / bits;
  int64_t rows = 1;
  for (int i = 0; i + 1 < nd; ++i) {
    rows *= x->shape[i];
    if (code->shape[i] != x->shape[i] || scale->shape[i] != x->shape[i] || mn->shape[i] != x->shape[i])
      return fail(BD_ERR_SHAPE, "leading dims of outputs must match x");
  }
  if (code->shape[nd - 1] * fpi != N || scale->shape[nd - 1] * 32 != N || mn->shape[nd - 1] * 32 != N)
    return fail(BD_ERR_SHAPE, "code must be [..,N*bits/32], scale/mn [..,N/32]");
  // outputs are written densely
  auto dense = [&](const bd_tensor* t) {
    int64_t s = 1;
    for (int i = nd - 1; i >= 0; --i) {
      if (t->shape[i] > 1 && t->stride[i] != s) return false;
      s *= t->shape[i];
    }
    return true;
  };
  if (!dense(code) || !dense(scale) || !dense(mn)) return fail(BD_ERR_STRIDE, "code, scale, mn must be contiguous");
  if (rows * N == 0) return BD_OK;
  int64_t l[3] = {1, 1, 1}, s[3] = {0, 0, 0};
  for (int i = 0; i + 1 < nd; ++i) { l[3 - (nd - 1) + i] = x->shape[i]; s[3 - (nd - 1) + i] = x->stride[i]; }
  const int64_t total = rows * (N / 32);
  const int threads = 128;
  const unsigned blocks = unsigned((total + threads - 1) / threads);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint32_t* cd = static_cast<uint32_t*>(code->data);
#define BD_PACK(T, BT)                                                                                         \
  if (bits == 2) kivi_pack_kernel<T, 2><<<blocks, threads, 0, st>>>(static_cast<const T*>(x->data), nd - 1, l[0], l[1], l[2], s[0], s[1], s[2], int(N), total, cd, static_cast<T*>(scale->data), static_cast<T*>(mn->data)); \
  else if (bits == 4) kivi_pack_kernel<T, 4><<<blocks, threads, 0, st>>>(static_cast<const T*>(x->data), nd - 1, l[0], l[1], l[2], s[0], s[1], s[2], int(N), total, cd, static_cast<T*>(scale->data), static_cast<T*>(mn->data)); \
  else kivi_pack_kernel<T, 8><<<blocks, threads, 0, st>>>(static_cast<const T*>(x->data), nd - 1, l[0], l[1], l[2], s[0], s[1], s[2], int(N), total, cd, static_cast<T*>(scale->data), static_cast<T*>(mn->data));
  if (x->dtype == BD_F16) { BD_PACK(__half, BD_F16) }
  else if (x->dtype == BD_BF16) { BD_PACK(__nv_bfloat16, BD_BF16) }
  else { BD_PACK(float, BD_F32) }
#undef BD_PACK
  return cuda_check(cudaGetLastError(), "kivi_pack_kernel launch");
}

int bd_kivi_append(const bd_tensor* k_new, const bd_tensor* v_new, int bits, int group_size, int64_t token_offset,
                   const bd_tensor* Kq, const bd_tensor* K_scale, const bd_tensor* K_mn, const bd_tensor* Vq,
                   const bd_tensor* V_scale, const bd_tensor* V_mn, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if (bits != 2 && bits != 4) return fail(BD_ERR_VALUE, "bits must be 2 or 4");
  if (group_size != 32) return fail(BD_ERR_UNSUPPORTED, "group_size must be 32");
  if ((rc = check_tensor(k_new, "k_new", 4)) || (rc = check_tensor(v_new, "v_new", 4, k_new->dtype)) ||
      (rc = check_tensor(Kq, "Kq", 4, BD_I32)) || (rc = check_tensor(K_scale, "K_scale", 4, BD_F16)) ||
      (rc = check_tensor(K_mn, "K_mn", 4, BD_F16)) || (rc = check_tensor(Vq, "Vq", 4, BD_I32)) ||
      (rc = check_tensor(V_scale, "V_scale", 4, BD_F16)) || (rc = check_tensor(V_mn, "V_mn", 4, BD_F16)))
    return rc;
  if (k_new->dtype != BD_F16 && k_new->dtype != BD_BF16 && k_new->dtype != BD_F32)
    return fail(BD_ERR_DTYPE, "k_new/v_new must be f16, bf16 or f32");
  const int64_t B = k_new->shape[0], Hk = k_new->shape[1], Tn = k_new->shape[2], D = k_new->shape[3];
  const int fpi = 32 / bits;
  for (int i = 0; i < 4; ++i)
    if (v_new->shape[i] != k_new->shape[i]) return fail(BD_ERR_SHAPE, "k_new and v_new shapes differ");
  if (Tn % 32 || D % 32) return fail(BD_ERR_SHAPE, "new tokens and head_dim must be multiples of 32");
  if (token_offset < 0 || token_offset % 32) return fail(BD_ERR_VALUE, "token_offset must be a non-negative multiple of 32");
  if ((Tn > 1 && (k_new->stride[3] != 1 || v_new->stride[3] != 1)))
    return fail(BD_ERR_STRIDE, "k_new/v_new channels must be contiguous");
  const int64_t end = token_offset + Tn;
  if (Kq->shape[0] != B || Kq->shape[1] != Hk || Kq->shape[2] != D || Kq->shape[3] * fpi < end)
    return fail(BD_ERR_SHAPE, "Kq must be [B,Hk,D,>= (offset+new)/fpi]");
  for (const bd_tensor* t : {K_scale, K_mn})
    if (t->shape[0] != B || t->shape[1] != Hk || t->shape[2] != D || t->shape[3] * 32 < end)
      return fail(BD_ERR_SHAPE, "K_scale/K_mn must be [B,Hk,D,>= (offset+new)/32]");
  if (Vq->shape[0] != B || Vq->shape[1] != Hk || Vq->shape[2] < end || Vq->shape[3] * fpi != D)
    return fail(BD_ERR_SHAPE, "Vq must be [B,Hk,>= offset+new,D/fpi]");
  for (const bd_tensor* t : {V_scale, V_mn})
    if (t->shape[0] != B || t->shape[1] != Hk || t->shape[2] < end || t->shape[3] * 32 != D)
      return fail(BD_ERR_SHAPE, "V_scale/V_mn must be [B,Hk,>= offset+new,D/32]");
  for (const bd_tensor* t : {Kq, K_scale, K_mn, Vq, V_scale, V_mn})
    if (t->shape[3] > 1 && t->stride[3] != 1) return fail(BD_ERR_STRIDE, "cache rows must be contiguous");
  if (B * Hk * Tn == 0) return BD_OK;
  AppendParams p{};
  p.k = k_new->data; p.k_sb = k_new->stride[0]; p.k_sh = k_new->stride[1]; p.k_st = k_new->stride[2];
  p.v = v_new->data; p.v_sb = v_new->stride[0]; p.v_sh = v_new->stride[1]; p.v_st = v_new->stride[2];
  p.in_dtype = k_new->dtype;
  p.B = int(B); p.Hk = int(Hk); p.Tn = int(Tn); p.D = int(D); p.t0 = token_offset;
  p.kq = static_cast<uint32_t*>(Kq->data); p.kq_sb = Kq->stride[0]; p.kq_sh = Kq->stride[1]; p.kq_sc = Kq->stride[2];
  p.ks = static_cast<__half*>(K_scale->data); p.ks_sb = K_scale->stride[0]; p.ks_sh = K_scale->stride[1]; p.ks_sc = K_scale->stride[2];
  p.km = static_cast<__half*>(K_mn->data); p.km_sb = K_mn->stride[0]; p.km_sh = K_mn->stride[1]; p.km_sc = K_mn->stride[2];
  p.vq = static_cast<uint32_t*>(Vq->data); p.vq_sb = Vq->stride[0]; p.vq_sh = Vq->stride[1]; p.vq_st = Vq->stride[2];
  p.vs = static_cast<__half*>(V_scale->data); p.vs_sb = V_scale->stride[0]; p.vs_sh = V_scale->stride[1]; p.vs_st = V_scale->stride[2];
  p.vm = static_cast<__half*>(V_mn->data); p.vm_sb = V_mn->stride[0]; p.vm_sh = V_mn->stride[1]; p.vm_st = V_mn->stride[2];
  const int64_t total = B * Hk * (Tn / 32) * D + B * Hk * Tn * (D / 32);
  const unsigned blocks = unsigned((total + 127) / 128);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (bits == 2) kivi_append_kernel<2><<<blocks, 128, 0, st>>>(p);
  else kivi_append_kernel<4><<<blocks, 128, 0, st>>>(p);
  return cuda_check(cudaGetLastError(), "kivi_append_kernel launch");
}

int bd_kivi_gemv_outer(int group_size, const bd_tensor* fA, const bd_tensor* qB, const bd_tensor* scales,
                       const bd_tensor* zeros, int bits, const bd_tensor* out, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if (bits != 2 && bits != 4 && bits != 8) return fail(BD_ERR_VALUE, "bits must be 2, 4 or 8");
  if (group_size <= 0) return fail(BD_ERR_VALUE, "group_size must be positive");
  if ((rc = check_tensor(fA, "fA", 4, BD_F16)) || (rc = check_tensor(qB, "qB", 4, BD_I32)) ||
      (rc = check_tensor(scales, "scales", 4, BD_F16)) || (rc = check_tensor(zeros, "zeros", 4, BD_F16)) ||
      (rc = check_tensor(out, "out", 4, BD_F16)))
    return rc;
  const int64_t B = fA->shape[0], Hq = fA->shape[1], M = fA->shape[2], K = fA->shape[3];
  const int64_t Hk = qB->shape[1], N = qB->shape[3] * (32 / bits);
  if (Hk <= 0 || Hq % Hk) return fail(BD_ERR_SHAPE, "fA heads must be a multiple of qB heads");
  if (qB->shape[0] != B || qB->shape[2] != K) return fail(BD_ERR_SHAPE, "qB must be [B,Hk,K,N*bits/32]");
  if (N % group_size) return fail(BD_ERR_SHAPE, "N must be a multiple of group_size");
  for (const bd_tensor* t : {scales, zeros})
    if (t->shape[0] != B || t->shape[1] != Hk || t->shape[2] != K || t->shape[3] * group_size != N)
      return fail(BD_ERR_SHAPE, "scales/zeros must be [B,Hk,K,N/group_size]");
  if (out->shape[0] != B || out->shape[1] != Hq || out->shape[2] != M || out->shape[3] != N)
    return fail(BD_ERR_SHAPE, "out must be [B,Hq,M,N]");
  if ((fA->stride[3] != 1 && K > 1) || (qB->stride[3] != 1 && qB->shape[3] > 1) || (scales->stride[3] != 1 && scales->shape[3] > 1) ||
      (zeros->stride[3] != 1 && zeros->shape[3] > 1) || (out->stride[3] != 1 && N > 1))
    return fail(BD_ERR_STRIDE, "innermost dims must be contiguous");
  if (B * Hq * M * N == 0) return BD_OK;
  GemvParams p{};
  p.fa = static_cast<const __half*>(fA->data); p.fa_sb = fA->stride[0]; p.fa_sh = fA->stride[1]; p.fa_sm = fA->stride[2];
  p.qb = static_cast<const uint32_t*>(qB->data); p.qb_sb = qB->stride[0]; p.qb_sh = qB->stride[1]; p.qb_sk = qB->stride[2];
  p.sc = static_cast<const __half*>(scales->data); p.sc_sb = scales->stride[0]; p.sc_sh = scales->stride[1]; p.sc_sk = scales->stride[2];
  p.zr = static_cast<const __half*>(zeros->data); p.zr_sb = zeros->stride[0]; p.zr_sh = zeros->stride[1]; p.zr_sk = zeros->stride[2];
  p.out = static_cast<__half*>(out->data); p.o_sb = out->stride[0]; p.o_sh = out->stride[1]; p.o_sm = out->stride[2];
  p.B = int(B); p.Hq = int(Hq); p.Hk = int(Hk); p.M = int(M); p.K = int(K); p.N = int(N); p.bits = bits; p.gs = group_size;
  dim3 grid(unsigned((N + 127) / 128), unsigned(B * Hq));
  kivi_gemv_kernel<<<grid, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return cuda_check(cudaGetLastError(), "kivi_gemv_kernel launch");
}

}  // extern "C"
