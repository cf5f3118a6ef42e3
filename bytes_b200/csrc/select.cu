// Top-k selection, sparse gather-attention and Quest page selection.
//
// References (saifmb0/bytes):
//   scores.topk(kb)                src/attention_kernels.py:1069,1262 (torch radix select)
//   select_topk('exact')           benchmarks/sparse_attention.py:287-309
//   sparse_gather_attn             src/attention_kernels.py:987-1059
//   attend_topk                    benchmarks/sparse_attention.py:367-387
//   _quest_select                  benchmarks/sparse_attention.py:328-364
//
// Top-k (one CTA per row): fp32 scores map to order-preserving u32 keys (-0 folded into
// +0). An MSB-first 8-bit radix select over the row (held in shared memory when it fits)
// finds the k-th key T and how many keys equal to T to keep; an ordered warp-ballot
// compaction then emits every key > T plus the lowest-index keys == T, in ascending index
// order. Ties are therefore broken by lower index, exactly like a stable descending sort.
// Optionally the k winners are bitonic-sorted by (key desc, index asc).
//
// The kernels of a selection chain (Quest bounds -> top-k -> page expansion -> gather, and
// scores -> top-k -> gather) are programmatic launches: each waits (griddepcontrol.wait)
// before touching global memory, so its CTAs are resident when the previous kernel ends.
// The one-CTA-per-SM top-k kernels for long rows are launched plainly.
#include "common.cuh"
#include "decode_shared.cuh"

#include <algorithm>
#include <type_traits>
#include <cmath>

namespace bd {
namespace {

constexpr int kTkThreads = 1024;
constexpr int kTkWarps = kTkThreads / 32;
constexpr int kSmemRowMax = 45 * 1024;  // keys held in shared memory up to this row length

__device__ __forceinline__ uint32_t f2key(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) == 0) u = 0;  // -0 == +0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

struct TopkParams {
  const float* scores; int64_t row_stride; int rows_per_b; int64_t b_stride;  // row r -> (r / rows_per_b, r % rows_per_b)
  int n, k;
  float* vals; int64_t v_rs;        // optional
  void* idx; int64_t i_rs; int idx64;
  int sorted;
};

// Block-wide exclusive scan of one value per warp (32 warps). Returns this warp's base
// and writes the total to *total. Uses red[] (32 ints).
__device__ __forceinline__ int warp_base_scan(int v, int* red, int* total) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int x = red[lane];
    int incl = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    red[lane] = incl - x;
    if (lane == 31) red[32] = incl;
  }
  __syncthreads();
  const int base = red[warp];
  *total = red[32];
  __syncthreads();
  return base;
}

// Block-wide exclusive scan of one int per thread (1024 threads); red[] holds 33 ints.
__device__ __forceinline__ int block_excl_scan(int v, int* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) red[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int x = red[lane];
    int wi = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    red[lane] = wi - x;
  }
  __syncthreads();
  const int r = red[warp] + incl - v;
  __syncthreads();
  return r;
}

// In a digit histogram of nb bins, find the digit holding the `remaining`-th largest key
// (digits scanned from nb-1 down) and the number of keys in higher digits. Thread t
// owns the bins nb-1-t*per .. nb-per-t*per. Results in *s_digit, *s_above.
__device__ __forceinline__ void find_digit(const int* hist, int nb, int remaining, int* red, int* s_digit,
                                           int* s_above) {
  const int per = nb > kTkThreads ? nb / kTkThreads : 1;
  const int d0 = nb - 1 - int(threadIdx.x) * per;
  int sum = 0;
  if (d0 >= 0)
    for (int j = 0; j < per; ++j) sum += hist[d0 - j];
  const int excl = block_excl_scan(sum, red);
  if (d0 >= 0 && excl < remaining && excl + sum >= remaining) {
    int acc = excl;
    for (int j = 0; j < per; ++j) {
      const int c = hist[d0 - j];
      if (acc + c >= remaining) { *s_digit = d0 - j; *s_above = acc; break; }
      acc += c;
    }
  }
  __syncthreads();
}

constexpr int kCandMax = 2048;  // candidates of the first 12-bit digit kept for the remaining digits
constexpr int kWarpCand = kCandMax / kTkWarps;  // candidate slots per warp

// Top-k for a row held in shared memory with 16-byte aligned float4 access (n % 4 == 0).
// One load pass builds a 12-bit histogram (bits 31..20 of the key); one filter pass copies
// the keys of the threshold digit (a few hundred for real-valued scores) with their
// indices; the remaining 20 bits (12 + 8) are resolved on those candidates only, or on the
// whole row if they overflow kCandMax. Selection and ordering rules as topk_kernel.
__global__ void __launch_bounds__(kTkThreads, 1) topk_fast_kernel(const TopkParams p) {
  griddep_wait();  // programmatic launch: the previous kernel's results are complete past here
  griddep_launch_dependents();
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ int red[33];
  __shared__ int s_digit, s_above, s_overflow;
  __shared__ int s_wcnt[kTkWarps];
  const int n = p.n, k = min(p.k, p.n), n4 = p.n >> 2;
  const int row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* src = p.scores + int64_t(row / p.rows_per_b) * p.b_stride + int64_t(row % p.rows_per_b) * p.row_stride;
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem);
  uint4* keys4 = reinterpret_cast<uint4*>(smem);
  int* hist = reinterpret_cast<int*>(smem + size_t(n) * 4);  // [4096]
  uint32_t* ck = reinterpret_cast<uint32_t*>(hist + 4096);     // [kCandMax], kWarpCand per warp
  if (k <= 0) return;

  // ---- load, keys to shared memory, 12-bit histogram
  if (threadIdx.x == 0) s_overflow = 0;
  for (int i = threadIdx.x; i < 4096; i += kTkThreads) hist[i] = 0;
  __syncthreads();
  {
    // eight 16-byte loads in flight per thread before any of them is consumed
    constexpr int U = 8;
    const float4* src4 = reinterpret_cast<const float4*>(src);
    for (int c0 = 0; c0 < n4; c0 += U * kTkThreads) {
      float4 x[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = c0 + u * kTkThreads + threadIdx.x;
        x[u] = i < n4 ? src4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = c0 + u * kTkThreads + threadIdx.x;
        if (i < n4) {
          const uint4 kk = make_uint4(f2key(x[u].x), f2key(x[u].y), f2key(x[u].z), f2key(x[u].w));
          keys4[i] = kk;
          atomicAdd(&hist[kk.x >> 20], 1); atomicAdd(&hist[kk.y >> 20], 1);
          atomicAdd(&hist[kk.z >> 20], 1); atomicAdd(&hist[kk.w >> 20], 1);
        }
      }
    }
  }
  __syncthreads();
  const bool take_all = k >= n;
  uint32_t prefix = 0, mask = 0;
  int remaining = k, eq_total = 0;
  if (!take_all) {
    find_digit(hist, 4096, remaining, red, &s_digit, &s_above);
    prefix = uint32_t(s_digit) << 20;
    mask = 0xfff00000u;
    remaining -= s_above;
    // ---- candidates: keys whose top 12 bits equal the threshold digit, appended to a
    // per-warp buffer of kWarpCand slots (no shared counter); any overflow sends the
    // remaining digits to the whole row
    {
      const unsigned lt = (1u << lane) - 1u;
      uint32_t* wck = ck + warp * kWarpCand;
      int wcnt = 0;  // warp-uniform
      for (int i0 = 0; i0 < n4; i0 += kTkThreads) {  // warp-uniform trip count
        const int i = i0 + threadIdx.x;
        const uint4 kk = i < n4 ? keys4[i] : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t kv[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const bool m = i < n4 && (kv[e] & mask) == prefix;
          const unsigned bm = __ballot_sync(0xffffffffu, m);
          const int pos = wcnt + __popc(bm & lt);
          if (m && pos < kWarpCand) wck[pos] = kv[e];
          wcnt += __popc(bm);
        }
      }
      if (lane == 0) {
        s_wcnt[warp] = wcnt;
        if (wcnt > kWarpCand) s_overflow = 1;
      }
    }
    __syncthreads();
    const bool in_cand = s_overflow == 0;
    // ---- remaining digits: bits 19..8 (12 bits), then 7..0 (8 bits)
#pragma unroll 1
    for (int pass = 0; pass < 2; ++pass) {
      const int shift = pass == 0 ? 8 : 0, nb = pass == 0 ? 4096 : 256;
      for (int i = threadIdx.x; i < nb; i += kTkThreads) hist[i] = 0;
      __syncthreads();
      if (in_cand) {
        for (int j = threadIdx.x; j < kCandMax; j += kTkThreads) {
          if (j % kWarpCand >= s_wcnt[j / kWarpCand]) continue;
          const uint32_t kk = ck[j];
          if ((kk & mask) == prefix) atomicAdd(&hist[(kk >> shift) & uint32_t(nb - 1)], 1);
        }
      } else {
        for (int j = threadIdx.x; j < n; j += kTkThreads) {
          const uint32_t kk = keys[j];
          if ((kk & mask) == prefix) atomicAdd(&hist[(kk >> shift) & uint32_t(nb - 1)], 1);
        }
      }
      __syncthreads();
      find_digit(hist, nb, remaining, red, &s_digit, &s_above);
      prefix |= uint32_t(s_digit) << shift;
      mask |= uint32_t(nb - 1) << shift;
      remaining -= s_above;
    }
    eq_total = hist[s_digit];  // keys equal to the full threshold (last digit's bin)
  }
  // threshold T = prefix; keep all keys > T and the `remaining` lowest-index keys == T.
  const uint32_t T = prefix;
  const int keep_eq = remaining;
  const unsigned lt = (1u << lane) - 1u;
  uint32_t* wk = reinterpret_cast<uint32_t*>(ck + kCandMax);
  const int kpow = p.sorted ? (k <= 1 ? 1 : 1 << (32 - __clz(k - 1))) : 0;
  int* wi = reinterpret_cast<int*>(wk + kpow);
  const int seg4 = (n4 + kTkWarps - 1) / kTkWarps;  // uint4 per warp segment
  const int s0 = min(n4, warp * seg4), s1 = min(n4, s0 + seg4);
  auto emit = [&](int o, uint32_t key, int ix) {
    if (p.sorted) {
      wk[o] = key;
      wi[o] = ix;
    } else {
      if (p.vals) p.vals[int64_t(row) * p.v_rs + o] = key2f(key);
      if (p.idx64) reinterpret_cast<int64_t*>(p.idx)[int64_t(row) * p.i_rs + o] = ix;
      else reinterpret_cast<int32_t*>(p.idx)[int64_t(row) * p.i_rs + o] = ix;
    }
  };
  if (take_all || keep_eq == eq_total) {
    // every key >= T is selected (exactly k of them): one count pass, one write pass
    int cnt = 0;
    for (int i = s0 + lane; i < s1; i += 32) {
      const uint4 x = keys4[i];
      cnt += (x.x >= T) + (x.y >= T) + (x.z >= T) + (x.w >= T);
    }
    cnt = __reduce_add_sync(0xffffffffu, cnt);
    int tot;
    int pos = warp_base_scan(cnt, red, &tot);
    for (int i0 = s0; i0 < s1; i0 += 32) {  // warp-uniform trip count
      const int i = i0 + lane;
      const uint4 x = i < s1 ? keys4[i] : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t kv[4] = {x.x, x.y, x.z, x.w};
      bool sel[4];
      unsigned bal[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        sel[e] = i < s1 && kv[e] >= T;
        bal[e] = __ballot_sync(0xffffffffu, sel[e]);
      }
      if ((bal[0] | bal[1] | bal[2] | bal[3]) == 0u) continue;
      int o = pos + __popc(bal[0] & lt) + __popc(bal[1] & lt) + __popc(bal[2] & lt) + __popc(bal[3] & lt);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (sel[e]) emit(o++, kv[e], 4 * i + e);
      pos += __popc(bal[0]) + __popc(bal[1]) + __popc(bal[2]) + __popc(bal[3]);
    }
  } else {

  // ---- general case (ties at T trimmed by index): ranks of the equal keys in index
  // order; warp w walks a contiguous segment, 4 keys per lane per step
  auto load4 = [&](int i, uint32_t* kv) {
    const uint4 x = i < s1 ? keys4[i] : make_uint4(0u, 0u, 0u, 0u);
    kv[0] = x.x; kv[1] = x.y; kv[2] = x.z; kv[3] = x.w;
  };
  int eq_cnt = 0;
  if (!take_all)
    for (int i0 = s0; i0 < s1; i0 += 32) {
      const int i = i0 + lane;
      uint32_t kv[4];
      load4(i, kv);
      int c = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) c += (i < s1 && kv[e] == T);
      eq_cnt += __reduce_add_sync(0xffffffffu, c);
    }
  int eq_total;
  const int eq_base = warp_base_scan(eq_cnt, red, &eq_total);
  // selection flags of a step: sel bit e of lane; returns the lane's selected count
  auto step_sel = [&](int i, const uint32_t* kv, int& eq_run, int* sel) {
    int eqf[4], eq_own = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) { eqf[e] = (i < s1 && kv[e] == T); eq_own += eqf[e]; }
    // equal keys before this lane in the step: inclusive scan of eq_own over lanes
    int incl = eq_own;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    int rank = eq_run + incl - eq_own;
    int cnt = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      sel[e] = i < s1 && (take_all || kv[e] > T || (eqf[e] && rank < keep_eq));
      rank += eqf[e];
      cnt += sel[e];
    }
    eq_run += __shfl_sync(0xffffffffu, incl, 31);
    return cnt;
  };
  int sel_cnt = 0;
  {
    int eq_run = eq_base;
    for (int i0 = s0; i0 < s1; i0 += 32) {
      const int i = i0 + lane;
      uint32_t kv[4];
      int sel[4];
      load4(i, kv);
      sel_cnt += __reduce_add_sync(0xffffffffu, step_sel(i, kv, eq_run, sel));
    }
  }
  int sel_total;
  const int sel_base = warp_base_scan(sel_cnt, red, &sel_total);
  {
    int eq_run = eq_base, pos = sel_base;
    for (int i0 = s0; i0 < s1; i0 += 32) {
      const int i = i0 + lane;
      uint32_t kv[4];
      int sel[4];
      load4(i, kv);
      const int c = step_sel(i, kv, eq_run, sel);
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      int o = pos + incl - c;
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (sel[e]) emit(o++, kv[e], 4 * i + e);
      pos += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  }  // general case
  if (!p.sorted) return;
  __syncthreads();
  // ---- bitonic sort of kpow (key desc, index asc); padding sorts last
  for (int i = k + threadIdx.x; i < kpow; i += kTkThreads) { wk[i] = 0u; wi[i] = 0x7fffffff; }
  __syncthreads();
  for (int size = 2; size <= kpow; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int t = threadIdx.x; t < kpow / 2; t += kTkThreads) {
        const int lo = 2 * t - (t & (stride - 1));
        const int hi = lo + stride;
        const bool desc_block = ((lo & size) == 0);
        const uint32_t ka = wk[lo], kb = wk[hi];
        const int ia = wi[lo], ib = wi[hi];
        const bool a_first = (ka > kb) || (ka == kb && ia < ib);
        if (a_first != desc_block) {
          wk[lo] = kb; wk[hi] = ka;
          wi[lo] = ib; wi[hi] = ia;
        }
      }
      __syncthreads();
    }
  }
  for (int o = threadIdx.x; o < k; o += kTkThreads) {
    if (p.vals) p.vals[int64_t(row) * p.v_rs + o] = key2f(wk[o]);
    if (p.idx64) reinterpret_cast<int64_t*>(p.idx)[int64_t(row) * p.i_rs + o] = wi[o];
    else reinterpret_cast<int32_t*>(p.idx)[int64_t(row) * p.i_rs + o] = wi[o];
  }
}

// ---- short rows (n <= kSmRowMax): one 256-thread CTA per row, each thread holding a
// contiguous run of up to kSmPer keys in registers. Four 8-bit MSB-first radix passes find
// the k-th key T and how many keys equal to T to keep; two block scans then give every
// selected key its output slot in index order (lower index first among equal keys), and
// sorted output is a bitonic sort of those k entries in shared memory.
constexpr int kSmThreads = 256;
constexpr int kSmWarps = kSmThreads / 32;
constexpr int kSmPer = 16;
constexpr int kSmRowMax = kSmThreads * kSmPer;
constexpr int kSmSortMax = 1024;  // largest k with sorted output on this path

// Exclusive scan of one int per thread over kSmWarps warps; *total receives the sum.
__device__ __forceinline__ int small_excl_scan(int v, int* red, int* total) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) red[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int x = lane < kSmWarps ? red[lane] : 0;
    int wi = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    if (lane < kSmWarps) red[lane] = wi - x;
    if (lane == kSmWarps - 1) red[32] = wi;
  }
  __syncthreads();
  const int r = red[warp] + incl - v;
  *total = red[32];
  __syncthreads();
  return r;
}

template <int PER>
__global__ void __launch_bounds__(kSmThreads, 4) topk_small_kernel(const TopkParams p) {
  griddep_wait();  // programmatic launch: the previous kernel's results are complete past here
  griddep_launch_dependents();
  extern __shared__ __align__(16) uint8_t smem[];  // sorted output: [kpow] keys, [kpow] indices
  __shared__ int hist[2][256];
  __shared__ int red[33];
  __shared__ int s_digit, s_above;
  const int row = blockIdx.x;
  const float* src = p.scores + int64_t(row / p.rows_per_b) * p.b_stride + int64_t(row % p.rows_per_b) * p.row_stride;
  const int n = p.n, k = min(p.k, p.n);
  if (k <= 0) return;
  const int i0 = int(threadIdx.x) * PER;  // this thread's run of PER positions
  uint32_t key[PER];
  const bool vec = (reinterpret_cast<uintptr_t>(src) & 15) == 0;
#pragma unroll
  for (int e = 0; e < PER; e += 4) {
    if (vec && i0 + e + 3 < n) {
      const float4 x = *reinterpret_cast<const float4*>(src + i0 + e);
      key[e] = f2key(x.x); key[e + 1] = f2key(x.y); key[e + 2] = f2key(x.z); key[e + 3] = f2key(x.w);
    } else {
#pragma unroll
      for (int u = 0; u < 4; ++u) key[e + u] = i0 + e + u < n ? f2key(src[i0 + e + u]) : 0u;
    }
  }
  // candidates of the digit passes: bit e set while key e matches the prefix found so far
  uint32_t cand = 0;
#pragma unroll
  for (int e = 0; e < PER; ++e) cand |= uint32_t(i0 + e < n) << e;
  const uint32_t valid_bits = cand;
  auto valid = [&](int e) { return (valid_bits >> e) & 1u; };

  // ---- radix select of the k-th largest key: per pass one shared histogram (two buffers,
  // each cleared right after its pass) and one warp that scans the 256 bins from the top
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t prefix = 0, mask = 0;
  int remaining = k;
  if (k < n) {
    hist[0][threadIdx.x] = 0;
    hist[1][threadIdx.x] = 0;
    __syncthreads();
#pragma unroll 1
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      int* h = hist[pass & 1];
#pragma unroll
      for (int e = 0; e < PER; ++e)
        if ((cand >> e) & 1u) atomicAdd(&h[(key[e] >> shift) & 255u], 1);
      __syncthreads();
      if (warp == 0) {
        // lane L owns digits 255-8L down to 248-8L
        int c[8], sum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          c[j] = h[255 - 8 * lane - j];
          sum += c[j];
        }
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        int acc = incl - sum;  // keys in higher digits
        if (acc < remaining && acc + sum >= remaining) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (acc + c[j] >= remaining) {
              s_digit = 255 - 8 * lane - j;
              s_above = acc;
              break;
            }
            acc += c[j];
          }
        }
      }
      __syncthreads();
      prefix |= uint32_t(s_digit) << shift;
      mask |= 0xffu << shift;
      remaining -= s_above;
      h[threadIdx.x] = 0;  // this buffer serves pass + 2, after the other buffer's barriers
#pragma unroll
      for (int e = 0; e < PER; ++e)
        if ((key[e] & mask) != prefix) cand &= ~(1u << e);
    }
  }
  // ---- keep every key above T and the first `remaining` keys equal to T (index order)
  int eq = 0;
#pragma unroll
  for (int e = 0; e < PER; ++e) eq += (k < n && valid(e) && key[e] == prefix) ? 1 : 0;
  int tot;
  int eq_rank = small_excl_scan(eq, red, &tot);
  uint32_t selbits = 0;
  int nsel = 0;
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    bool sel = false;
    if (valid(e)) {
      if (k >= n || key[e] > prefix) sel = true;
      else if (key[e] == prefix) sel = eq_rank++ < remaining;
    }
    selbits |= uint32_t(sel) << e;
    nsel += sel;
  }
  int pos = small_excl_scan(nsel, red, &tot);
  uint32_t* wk = reinterpret_cast<uint32_t*>(smem);
  int kpow = 1;
  while (kpow < max(k, 1)) kpow <<= 1;
  int* wi = reinterpret_cast<int*>(smem + size_t(kpow) * 4);
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    if (!((selbits >> e) & 1u)) continue;
    const int idx = i0 + e;
    if (p.sorted) {
      wk[pos] = key[e];
      wi[pos] = idx;
    } else {
      if (p.vals) p.vals[int64_t(row) * p.v_rs + pos] = key2f(key[e]);
      if (p.idx64) reinterpret_cast<int64_t*>(p.idx)[int64_t(row) * p.i_rs + pos] = idx;
      else reinterpret_cast<int32_t*>(p.idx)[int64_t(row) * p.i_rs + pos] = idx;
    }
    ++pos;
  }
  if (!p.sorted) return;
  for (int i = k + threadIdx.x; i < kpow; i += kSmThreads) { wk[i] = 0u; wi[i] = 0x7fffffff; }
  __syncthreads();
  auto before = [](uint32_t ka, int ia, uint32_t kb, int ib) { return ka > kb || (ka == kb && ia < ib); };
  if (kpow <= 128) {
    // ---- one warp sorts in registers: element i = lane + 32r (r < E), bitonic network
    // (key desc, index asc); pairs 32 or more apart sit in one lane, closer ones meet by
    // shuffle. Padding (key 0, largest index) sorts last.
    if (warp != 0) return;
    const int E = (kpow + 31) / 32;
    uint32_t kk[4];
    int ii[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = lane + 32 * r;
      const bool in = r < E && i < kpow;
      kk[r] = in ? wk[i] : 0u;
      ii[r] = in ? wi[i] : 0x7fffffff;
    }
    for (int size = 2; size <= kpow; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        if (stride >= 32) {
          const int rs = stride >> 5;
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            if (r >= E || (r & rs)) continue;
            const int r2 = r | rs;
            const int i = lane + 32 * r;
            const bool desc = (i & size) == 0;
            if (before(kk[r], ii[r], kk[r2], ii[r2]) != desc) {
              const uint32_t tk = kk[r]; kk[r] = kk[r2]; kk[r2] = tk;
              const int ti = ii[r]; ii[r] = ii[r2]; ii[r2] = ti;
            }
          }
        } else {
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            if (r >= E) continue;  // warp-uniform
            const int i = lane + 32 * r;
            const uint32_t pk = __shfl_xor_sync(0xffffffffu, kk[r], stride);
            const int pi = __shfl_xor_sync(0xffffffffu, ii[r], stride);
            const bool lo = (lane & stride) == 0;
            const bool desc = (i & size) == 0;
            // the lower element of the pair keeps the one that comes first in this block's order
            const bool mine_first = before(kk[r], ii[r], pk, pi);
            const bool keep = (lo == desc) ? mine_first : !mine_first;
            if (!keep) { kk[r] = pk; ii[r] = pi; }
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int o = lane + 32 * r;
      if (r >= E || o >= k) continue;
      if (p.vals) p.vals[int64_t(row) * p.v_rs + o] = key2f(kk[r]);
      if (p.idx64) reinterpret_cast<int64_t*>(p.idx)[int64_t(row) * p.i_rs + o] = ii[r];
      else reinterpret_cast<int32_t*>(p.idx)[int64_t(row) * p.i_rs + o] = ii[r];
    }
    return;
  }
  // ---- bitonic sort of kpow entries in shared memory (key desc, index asc); padding last
  for (int size = 2; size <= kpow; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int t = threadIdx.x; t < kpow / 2; t += kSmThreads) {
        const int lo = 2 * t - (t & (stride - 1));
        const int hi = lo + stride;
        const bool desc_block = ((lo & size) == 0);
        const uint32_t ka = wk[lo], kb = wk[hi];
        const int ia = wi[lo], ib = wi[hi];
        const bool a_first = (ka > kb) || (ka == kb && ia < ib);
        if (a_first != desc_block) {
          wk[lo] = kb; wk[hi] = ka;
          wi[lo] = ib; wi[hi] = ia;
        }
      }
      __syncthreads();
    }
  }
  for (int o = threadIdx.x; o < k; o += kSmThreads) {
    if (p.vals) p.vals[int64_t(row) * p.v_rs + o] = key2f(wk[o]);
    if (p.idx64) reinterpret_cast<int64_t*>(p.idx)[int64_t(row) * p.i_rs + o] = wi[o];
    else reinterpret_cast<int32_t*>(p.idx)[int64_t(row) * p.i_rs + o] = wi[o];
  }
}

template <bool SMEM_ROW>
__global__ void __launch_bounds__(kTkThreads, 1) topk_kernel(const TopkParams p) {
  griddep_wait();  // programmatic launch: the previous kernel's results are complete past here
  griddep_launch_dependents();
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ int hist[256];
  __shared__ int red[33];
  __shared__ uint32_t s_prefix;
  __shared__ int s_remaining;
  const int row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* src = p.scores + int64_t(row / p.rows_per_b) * p.b_stride + int64_t(row % p.rows_per_b) * p.row_stride;
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem);
  const int n = p.n, k = min(p.k, p.n);
  auto key_at = [&](int i) -> uint32_t { return SMEM_ROW ? keys[i] : f2key(src[i]); };

  // ---- load + first-digit histogram
  for (int i = threadIdx.x; i < 256; i += kTkThreads) hist[i] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += kTkThreads) {
    const uint32_t kk = f2key(src[i]);
    if (SMEM_ROW) keys[i] = kk;
    atomicAdd(&hist[kk >> 24], 1);
  }
  __syncthreads();

  uint32_t prefix = 0, mask = 0;
  int remaining = k;
  if (k < n) {
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      if (pass > 0) {
        for (int i = threadIdx.x; i < 256; i += kTkThreads) hist[i] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += kTkThreads) {
          const uint32_t kk = key_at(i);
          if ((kk & mask) == prefix) atomicAdd(&hist[(kk >> shift) & 255], 1);
        }
        __syncthreads();
      }
      if (warp == 0) {
        // lane l owns digits 255-8l .. 248-8l (descending)
        int c[8], sum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) { c[j] = hist[255 - 8 * lane - j]; sum += c[j]; }
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        const int excl = incl - sum;
        const bool here = excl < remaining && incl >= remaining;
        if (here) {
          int acc = excl, d = 0;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (acc + c[j] >= remaining) { d = 255 - 8 * lane - j; break; }
            acc += c[j];
          }
          s_prefix = prefix | (uint32_t(d) << shift);
          s_remaining = remaining - acc;
        }
      }
      __syncthreads();
      prefix = s_prefix;
      remaining = s_remaining;
      mask |= 255u << shift;
      __syncthreads();
    }
  }
  // threshold T = prefix; keep all keys > T and the `remaining` lowest-index keys == T.
  const uint32_t T = prefix;
  const int keep_eq = remaining;
  const bool take_all = k >= n;

  // ---- ordered compaction: warp w walks a contiguous segment
  const int seg = ((n + kTkWarps - 1) / kTkWarps + 31) & ~31;
  const int s0 = min(n, warp * seg), s1 = min(n, s0 + seg);
  const unsigned lt = (1u << lane) - 1u;
  int eq_cnt = 0;
  if (!take_all)
    for (int i0 = s0; i0 < s1; i0 += 32) {
      const int i = i0 + lane;
      const bool eq = i < s1 && key_at(i) == T;
      eq_cnt += __popc(__ballot_sync(0xffffffffu, eq));
    }
  int eq_total;
  const int eq_base = warp_base_scan(eq_cnt, red, &eq_total);
  int sel_cnt = 0;
  {
    int eq_run = eq_base;
    for (int i0 = s0; i0 < s1; i0 += 32) {
      const int i = i0 + lane;
      const uint32_t kk = i < s1 ? key_at(i) : 0u;
      const bool eq = i < s1 && kk == T;
      const unsigned eb = __ballot_sync(0xffffffffu, eq);
      const int rank = eq_run + __popc(eb & lt);
      const bool sel = i < s1 && (take_all || kk > T || (eq && rank < keep_eq));
      sel_cnt += __popc(__ballot_sync(0xffffffffu, sel));
      eq_run += __popc(eb);
    }
  }
  int sel_total;
  const int sel_base = warp_base_scan(sel_cnt, red, &sel_total);
  // winners go to shared memory (after the row keys) as (key, index) pairs when sorting,
  // else straight to the outputs in index order
  uint32_t* wk = reinterpret_cast<uint32_t*>(smem + (SMEM_ROW ? size_t(n) * 4 : 0));
  const int kpow = p.sorted ? (k <= 1 ? 1 : 1 << (32 - __clz(k - 1))) : 0;
  int* wi = reinterpret_cast<int*>(wk + kpow);
  {
    int eq_run = eq_base, pos = sel_base;
    for (int i0 = s0; i0 < s1; i0 += 32) {
      const int i = i0 + lane;
      const uint32_t kk = i < s1 ? key_at(i) : 0u;
      const bool eq = i < s1 && kk == T;
      const unsigned eb = __ballot_sync(0xffffffffu, eq);
      const int rank = eq_run + __popc(eb & lt);
      const bool sel = i < s1 && (take_all || kk > T || (eq && rank < keep_eq));
      const unsigned sb = __ballot_sync(0xffffffffu, sel);
      if (sel) {
        const int o = pos + __popc(sb & lt);
        if (p.sorted) {
          wk[o] = kk;
          wi[o] = i;
        } else {
          if (p.vals) p.vals[int64_t(row) * p.v_rs + o] = key2f(kk);
          if (p.idx64) reinterpret_cast<int64_t*>(p.idx)[int64_t(row) * p.i_rs + o] = i;
          else reinterpret_cast<int32_t*>(p.idx)[int64_t(row) * p.i_rs + o] = i;
        }
      }
      pos += __popc(sb);
      eq_run += __popc(eb);
    }
  }
  if (!p.sorted) return;
  __syncthreads();
  // ---- bitonic sort of kpow (key desc, index asc); padding sorts last
  for (int i = k + threadIdx.x; i < kpow; i += kTkThreads) { wk[i] = 0u; wi[i] = 0x7fffffff; }
  __syncthreads();
  for (int size = 2; size <= kpow; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int t = threadIdx.x; t < kpow / 2; t += kTkThreads) {
        const int lo = 2 * t - (t & (stride - 1));
        const int hi = lo + stride;
        const bool desc_block = ((lo & size) == 0);  // first half of each block sorts "before"
        const uint32_t ka = wk[lo], kb = wk[hi];
        const int ia = wi[lo], ib = wi[hi];
        // "a before b" if key larger, or equal key and smaller index
        const bool a_first = (ka > kb) || (ka == kb && ia < ib);
        if (a_first != desc_block) {
          wk[lo] = kb; wk[hi] = ka;
          wi[lo] = ib; wi[hi] = ia;
        }
      }
      __syncthreads();
    }
  }
  for (int o = threadIdx.x; o < k; o += kTkThreads) {
    if (p.vals) p.vals[int64_t(row) * p.v_rs + o] = key2f(wk[o]);
    if (p.idx64) reinterpret_cast<int64_t*>(p.idx)[int64_t(row) * p.i_rs + o] = wi[o];
    else reinterpret_cast<int32_t*>(p.idx)[int64_t(row) * p.i_rs + o] = wi[o];
  }
}

// ------------------------------------------------------------------ gather-attend
constexpr int kGatherChunk = 1024;  // split positions staged in shared memory at a time

struct GatherParams {
  const void* q; int64_t q_sb, q_sh; int q_dtype;
  const uint8_t* k; int64_t k_sb, k_sh, k_ss;
  const uint8_t* v; int64_t v_sb, v_sh, v_ss;
  const void* idx; int64_t i_sb, i_sh; int idx64;
  int B, Hq, Hk, G, S, kb;
  float scaling;
  int rows_per_split, nsplit;
  float* part_m; float* part_l; float* part_o;  // split partials (or, with one split, the exported m, l, o)
  void* out; int out_dtype; int64_t o_sb, o_sh;  // one split and a final output: written directly
};

// key/value element kinds of the gather (fp8 e4m3, bf16, f16, fp32), widened to fp32
enum GatherKv { kGvBf16 = 0, kGvFp8, kGvF16, kGvF32 };

template <int D, int KV>
__global__ void __launch_bounds__(128) gather_attn_kernel(const GatherParams p) {
  constexpr bool FP8 = KV == kGvFp8;
  griddep_wait();  // programmatic launch: the previous kernel's results are complete past here
  griddep_launch_dependents();  // the combine queued behind may start launching (it waits for this grid)
  constexpr int CPL = D / 8;  // channels per lane (8 lanes per row)
  constexpr int ELT = FP8 ? 1 : (KV == kGvF32 ? 4 : 2);
  __shared__ float red_m[16], red_l[16];
  __shared__ float red_o[16][D];
  const int split = blockIdx.x, hq = blockIdx.y, b = blockIdx.z;
  const int hk = hq / p.G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane >> 3, sub = lane & 7;  // 4 row groups of 8 lanes per warp
  const int gid = warp * 4 + grp;             // 16 row groups per CTA
  float qv[CPL];
  {
    const int64_t qo = int64_t(b) * p.q_sb + int64_t(hq) * p.q_sh + sub * CPL;
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      float x;
      if (p.q_dtype == BD_BF16) x = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.q)[qo + c]);
      else if (p.q_dtype == BD_F16) x = __half2float(reinterpret_cast<const __half*>(p.q)[qo + c]);
      else x = reinterpret_cast<const float*>(p.q)[qo + c];
      qv[c] = x;
    }
  }
  const uint8_t* kb_ = p.k + (int64_t(b) * p.k_sb + int64_t(hk) * p.k_sh) * ELT + sub * CPL * ELT;
  const uint8_t* vb_ = p.v + (int64_t(b) * p.v_sb + int64_t(hk) * p.v_sh) * ELT + sub * CPL * ELT;
  const int r_begin = split * p.rows_per_split;
  const int r_end = min(p.kb, r_begin + p.rows_per_split);
  float m = -INFINITY, l = 0.f, acc[CPL];
#pragma unroll
  for (int c = 0; c < CPL; ++c) acc[c] = 0.f;
  auto row_index = [&](int r) -> int64_t {
    const int64_t off = int64_t(b) * p.i_sb + int64_t(hq) * p.i_sh + r;
    return p.idx64 ? reinterpret_cast<const int64_t*>(p.idx)[off] : int64_t(reinterpret_cast<const int32_t*>(p.idx)[off]);
  };
  constexpr int WPL = CPL * ELT / 4;  // 32-bit words per lane per row (1, 2, 4 or 8)
  // one row's key and value words of this lane (zeros for a masked row)
  auto load_row = [&](int t, uint32_t (&kw)[WPL], uint32_t (&vw)[WPL]) {
#pragma unroll
    for (int w = 0; w < WPL; ++w) kw[w] = vw[w] = 0u;
    if (t < 0) return;
    const uint8_t* kr = kb_ + int64_t(t) * p.k_ss * ELT;
    const uint8_t* vr = vb_ + int64_t(t) * p.v_ss * ELT;
    if (WPL == 1) {
      kw[0] = __ldg(reinterpret_cast<const uint32_t*>(kr));
      vw[0] = __ldg(reinterpret_cast<const uint32_t*>(vr));
    } else if (WPL == 2) {
      const uint2 a = __ldg(reinterpret_cast<const uint2*>(kr)), c = __ldg(reinterpret_cast<const uint2*>(vr));
      kw[0] = a.x; kw[1] = a.y; vw[0] = c.x; vw[1] = c.y;
    } else {
#pragma unroll
      for (int u = 0; u < WPL / 4; ++u) {
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(kr) + u), c = __ldg(reinterpret_cast<const uint4*>(vr) + u);
        kw[4 * u] = a.x; kw[4 * u + 1] = a.y; kw[4 * u + 2] = a.z; kw[4 * u + 3] = a.w;
        vw[4 * u] = c.x; vw[4 * u + 1] = c.y; vw[4 * u + 2] = c.z; vw[4 * u + 3] = c.w;
      }
    }
  };
  // dot product with q (8-lane group reduction) and online-softmax update for one row
  auto consume = [&](bool ok, const uint32_t (&kw)[WPL], const uint32_t (&vw)[WPL]) {
    float kf[CPL], vf[CPL];
#pragma unroll
    for (int w = 0; w < WPL; ++w) {
      if (FP8) {
        const uint32_t k01 = e4m3x2_to_f16x2(kw[w]), k23 = e4m3x2_to_f16x2(kw[w] >> 16);
        const uint32_t v01 = e4m3x2_to_f16x2(vw[w]), v23 = e4m3x2_to_f16x2(vw[w] >> 16);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&k01));
        const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&k23));
        const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&v01));
        const float2 e = __half22float2(*reinterpret_cast<const __half2*>(&v23));
        kf[4 * w] = a.x; kf[4 * w + 1] = a.y; kf[4 * w + 2] = c.x; kf[4 * w + 3] = c.y;
        vf[4 * w] = d.x; vf[4 * w + 1] = d.y; vf[4 * w + 2] = e.x; vf[4 * w + 3] = e.y;
      } else if (KV == kGvF32) {
        kf[w] = __uint_as_float(kw[w]);
        vf[w] = __uint_as_float(vw[w]);
      } else if (KV == kGvF16) {
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&kw[w]));
        const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&vw[w]));
        kf[2 * w] = a.x; kf[2 * w + 1] = a.y;
        vf[2 * w] = c.x; vf[2 * w + 1] = c.y;
      } else {
        kf[2 * w] = __uint_as_float(kw[w] << 16);
        kf[2 * w + 1] = __uint_as_float(kw[w] & 0xffff0000u);
        vf[2 * w] = __uint_as_float(vw[w] << 16);
        vf[2 * w + 1] = __uint_as_float(vw[w] & 0xffff0000u);
      }
    }
    float sdot = 0.f;
#pragma unroll
    for (int c = 0; c < CPL; ++c) sdot = fmaf(qv[c], kf[c], sdot);
    sdot += __shfl_xor_sync(0xffffffffu, sdot, 1);
    sdot += __shfl_xor_sync(0xffffffffu, sdot, 2);
    sdot += __shfl_xor_sync(0xffffffffu, sdot, 4);
    if (!ok) return;  // masked position: contributes nothing (uniform within the 8-lane group)
    sdot *= p.scaling;
    const float mn = fmaxf(m, sdot);
    const float alpha = __expf(m - mn);
    const float pw = __expf(sdot - mn);
    l = l * alpha + pw;
#pragma unroll
    for (int c = 0; c < CPL; ++c) acc[c] = fmaf(pw, vf[c], acc[c] * alpha);
    m = mn;
  };
  // The split's positions come into shared memory a chunk at a time (one coalesced read;
  // out-of-range or negative positions become -1), then every 8-lane group takes four rows
  // per step (rows i, i + 16, i + 32, i + 48), all four rows' loads in flight before any
  // is used.
  __shared__ int s_pos[kGatherChunk];
  for (int c0 = r_begin; c0 < r_end; c0 += kGatherChunk) {
    const int n = min(kGatherChunk, r_end - c0);
    __syncthreads();  // the previous chunk's readers are done
    for (int i = threadIdx.x; i < n; i += 128) {
      const int64_t t = row_index(c0 + i);
      s_pos[i] = (t >= 0 && t < p.S) ? int(t) : -1;
    }
    __syncthreads();
    // all four 8-lane row groups of a warp iterate together (the shuffles need every lane
    // of the warp); a group whose row is past the chunk is predicated off
    for (int i0 = warp * 4; i0 < n; i0 += 64) {
      const int ia = i0 + grp, ib = ia + 16, ic = ia + 32, id = ia + 48;
      const int ta = ia < n ? s_pos[ia] : -1, tb = ib < n ? s_pos[ib] : -1;
      const int tc = ic < n ? s_pos[ic] : -1, td = id < n ? s_pos[id] : -1;
      uint32_t ka[WPL], va[WPL], kb2[WPL], vb2[WPL], kc[WPL], vc[WPL], kd[WPL], vd[WPL];
      load_row(ta, ka, va);
      load_row(tb, kb2, vb2);
      load_row(tc, kc, vc);
      load_row(td, kd, vd);
      consume(ta >= 0, ka, va);
      consume(tb >= 0, kb2, vb2);
      consume(tc >= 0, kc, vc);
      consume(td >= 0, kd, vd);
    }
  }
  // merge the 16 row groups
  if (sub == 0) { red_m[gid] = m; red_l[gid] = l; }
#pragma unroll
  for (int c = 0; c < CPL; ++c) red_o[gid][sub * CPL + c] = acc[c];
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += 128) {
    float M = -INFINITY;
#pragma unroll
    for (int i = 0; i < 16; ++i) M = fmaxf(M, red_m[i]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float f = M == -INFINITY ? 0.f : __expf(red_m[i] - M);
      L += red_l[i] * f;
      O += red_o[i][c] * f;
    }
    if (p.out) {  // one split: the final output, no combine
      const int64_t off = int64_t(b) * p.o_sb + int64_t(hq) * p.o_sh + c;
      const float x = O / L;
      if (p.out_dtype == BD_BF16) reinterpret_cast<__nv_bfloat16*>(p.out)[off] = __float2bfloat16_rn(x);
      else if (p.out_dtype == BD_F16) reinterpret_cast<__half*>(p.out)[off] = __float2half_rn(x);
      else reinterpret_cast<float*>(p.out)[off] = x;
      continue;
    }
    const int64_t pi = (int64_t(b) * p.Hq + hq) * p.nsplit + split;
    p.part_o[pi * D + c] = O;
    if (c == 0) { p.part_m[pi] = M; p.part_l[pi] = L; }
  }
}

// ------------------------------------------------------------------ Quest
template <typename T>
__global__ void quest_minmax_kernel(const T* __restrict__ k, int64_t s_b, int64_t s_h, int64_t s_s, int Hk, int S,
                                    int D, int page, int np, T* __restrict__ kmin, T* __restrict__ kmax,
                                    int64_t m_sb, int64_t m_sh, int64_t m_sp) {
  const int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;  // (b, h, page, d)
  const int64_t total = int64_t(gridDim.y) * Hk * np * D;
  (void)total;
  const int b = blockIdx.y;
  if (gid >= int64_t(Hk) * np * D) return;
  const int d = int(gid % D);
  const int64_t r = gid / D;
  const int pg = int(r % np), h = int(r / np);
  const T* src = k + int64_t(b) * s_b + int64_t(h) * s_h + d;
  const int t0 = pg * page, t1 = min(S, t0 + page);
  float lo = INFINITY, hi = -INFINITY;
  for (int t = t0; t < t1; ++t) {
    const float x = to_f32<T>(src[int64_t(t) * s_s]);
    lo = fminf(lo, x);
    hi = fmaxf(hi, x);
  }
  const int64_t o = int64_t(b) * m_sb + int64_t(h) * m_sh + int64_t(pg) * m_sp + d;
  kmin[o] = from_f32<T>(lo);
  kmax[o] = from_f32<T>(hi);
}

// bound[b,hq,p] = scaling * sum_d max(q_d*kmin_pd, q_d*kmax_pd); pages >= force_from -> +inf
// (the reference's fp32 bound, benchmarks/sparse_attention.py:342-345). Page metadata MT is
// bf16, f16 or fp32 (the key dtype), read unrounded; 64 pages per CTA (32 for fp32 rows).
constexpr int kQPages = 64;  // pages per CTA (one thread each) for 16-bit metadata

template <typename MT>
__device__ __forceinline__ float meta_f32(const uint8_t* p) {
  if constexpr (sizeof(MT) == 4) return *reinterpret_cast<const float*>(p);
  else return to_f32<MT>(*reinterpret_cast<const MT*>(p));
}

template <int D, typename MT>
__global__ void __launch_bounds__(kQPages) quest_bounds_kernel(const void* q, int q_dtype, int64_t q_sb, int64_t q_sh,
                                                         const MT* kmin, const MT* kmax,
                                                         int64_t m_sb, int64_t m_sh, int64_t m_sp, int Hq, int Hk,
                                                         int np, float scaling, int force_from, float* bounds) {
  griddep_wait();  // programmatic launch: the previous kernel's results are complete past here
  griddep_launch_dependents();
  constexpr int ES = int(sizeof(MT));
  constexpr int NP = ES == 4 ? kQPages / 2 : kQPages;  // pages per CTA
  constexpr int PITCH = D * ES + 16;
  constexpr int EPC = 16 / ES;  // elements per 16-byte chunk
  __shared__ __align__(16) uint8_t sm[2][NP * PITCH];
  const int b = blockIdx.z, hk = blockIdx.y, p0 = blockIdx.x * NP;
  const int G = Hq / Hk;
  const int npg = min(NP, np - p0);
  // stage the pages' min and max rows (padded pitch: conflict-free 16-byte reads)
  for (int c = threadIdx.x; c < npg * (D / EPC); c += NP) {
    const int r = c / (D / EPC), cc = c % (D / EPC);
    const int64_t go = int64_t(b) * m_sb + int64_t(hk) * m_sh + int64_t(p0 + r) * m_sp + cc * EPC;
    cp_async16(smem_u32(&sm[0][r * PITCH + cc * 16]), kmin + go, 16);
    cp_async16(smem_u32(&sm[1][r * PITCH + cc * 16]), kmax + go, 16);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  const int r = threadIdx.x;
  if (r >= npg) return;
  const int pg = p0 + r;
  for (int h0 = 0; h0 < G; h0 += 4) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int d = 0; d < D; ++d) {
      const float mnv = meta_f32<MT>(&sm[0][r * PITCH + d * ES]);
      const float mxv = meta_f32<MT>(&sm[1][r * PITCH + d * ES]);
#pragma unroll
      for (int hh = 0; hh < 4; ++hh) {
        if (h0 + hh >= G) break;
        const int64_t qi = int64_t(b) * q_sb + int64_t(hk * G + h0 + hh) * q_sh + d;
        float qd;
        if (q_dtype == BD_BF16) qd = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(q)[qi]);
        else if (q_dtype == BD_F16) qd = __half2float(reinterpret_cast<const __half*>(q)[qi]);
        else qd = reinterpret_cast<const float*>(q)[qi];
        acc[hh] += fmaxf(__fmul_rn(qd, mnv), __fmul_rn(qd, mxv));
      }
    }
#pragma unroll
    for (int hh = 0; hh < 4; ++hh) {
      if (h0 + hh >= G) break;
      const float v = pg >= force_from ? INFINITY : acc[hh] * scaling;
      bounds[(int64_t(b) * Hq + hk * G + h0 + hh) * np + pg] = v;
    }
  }
}

// Tensor-core form of the same bound for a bf16 query. Since max_pd >= min_pd,
//   max(q_d*min_pd, q_d*max_pd) = q+_d*max_pd + q-_d*min_pd   (q+ = max(q,0), q- = min(q,0)),
// so the bounds of a page tile are one GEMM: [max_p | min_p] (pages x 2D, bf16) times
// [q+ ; q-] (2D x heads, bf16, exact), fp32 accumulate -- mma.sync m16n8k16, 16 pages per
// warp, 8 heads per CTA. The page rows stream through a padded shared-memory tile
// (conflict-free ldmatrix); bytes per page and KV head: 4*D.
constexpr int kQmPages = 64;  // pages per CTA (4 warps x 16)

struct QuestMmaParams {
  const __nv_bfloat16* q; int64_t q_sb, q_sh;
  const __nv_bfloat16* kmin; const __nv_bfloat16* kmax; int64_t m_sb, m_sh, m_sp;
  int Hq, Hk, G, head_chunks, np, force_from;
  int blocks_per_cta;  // 64-page blocks each CTA streams
  float scaling;
  float* bounds;
};

// One CTA streams `blocks_per_cta` consecutive blocks of 64 pages of one (b, KV head,
// head chunk) through a two-stage cp.async pipeline (the next block's [max | min] rows load
// while this one's bounds are computed); the query fragments are built once per CTA.
template <int D>
__global__ void __launch_bounds__(128) quest_bounds_mma_kernel(const QuestMmaParams p) {
  griddep_wait();  // programmatic launch: the previous kernel's results are complete past here
  griddep_launch_dependents();
  constexpr int ROWB = 4 * D;        // [max | min] bf16 bytes per page
  constexpr int PITCH = ROWB + 16;   // padded row
  constexpr int CH = ROWB / 16;      // 16-byte chunks per page
  constexpr int KSTEPS = 2 * D / 16;
  constexpr int STAGE = kQmPages * PITCH;
  extern __shared__ __align__(16) uint8_t sm[];  // [2 stages][64 pages][PITCH]
  const int b = blockIdx.z, hk = blockIdx.y / p.head_chunks, chunk = blockIdx.y % p.head_chunks;
  const int blk0 = blockIdx.x * p.blocks_per_cta;
  const int nblk = min(p.blocks_per_cta, (p.np + kQmPages - 1) / kQmPages - blk0);
  if (nblk <= 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int64_t mbase = int64_t(b) * p.m_sb + int64_t(hk) * p.m_sh;
  auto load_block = [&](int i, int stage) {
    const int p0 = (blk0 + i) * kQmPages;
    const int npg = min(kQmPages, p.np - p0);
    for (int c = threadIdx.x; c < kQmPages * CH; c += 128) {
      const int r = c / CH, cc = c % CH;
      const bool ok = r < npg;
      const __nv_bfloat16* src = (cc < CH / 2 ? p.kmax : p.kmin) + mbase + int64_t(ok ? p0 + r : 0) * p.m_sp +
                                 (cc % (CH / 2)) * 8;
      cp_async16(smem_u32(sm + stage * STAGE + r * PITCH + cc * 16), src, ok ? 16 : 0);
    }
  };
  load_block(0, 0);
  cp_async_commit();
  // B fragments: head n = g of this chunk; k < D -> q+ (max rows), k >= D -> q- (min rows)
  const int h = chunk * 8 + g;
  const bool hv = h < p.G;
  const __nv_bfloat16* qr = p.q + int64_t(b) * p.q_sb + int64_t(hk * p.G + (hv ? h : 0)) * p.q_sh;
  uint32_t bq[KSTEPS][2];
#pragma unroll
  for (int kk = 0; kk < KSTEPS; ++kk)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int k = kk * 16 + 8 * e + 2 * tq;
      const int ch = k < D ? k : k - D;
      uint32_t w = hv ? *reinterpret_cast<const uint32_t*>(qr + ch) : 0u;
      __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162*>(&w);
      const __nv_bfloat162 z = __float2bfloat162_rn(0.f);
      x = k < D ? __hmax2(x, z) : __hmin2(x, z);
      bq[kk][e] = *reinterpret_cast<uint32_t*>(&x);
    }
  for (int i = 0; i < nblk; ++i) {
    cp_async_wait<0>();
    __syncthreads();  // block i landed; the stage block i+1 goes to was read last round
    if (i + 1 < nblk) load_block(i + 1, (i + 1) & 1);
    cp_async_commit();
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t arow = smem_u32(sm + (i & 1) * STAGE + (warp * 16 + (lane & 15)) * PITCH + (lane >> 4) * 16);
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      uint32_t a0, a1, a2, a3;
      ldmatrix_x4(a0, a1, a2, a3, arow + kk * 32);
      mma_bf16(acc, a0, a1, a2, a3, bq[kk][0], bq[kk][1]);
    }
    // acc: (page 16w+g, heads 2tq, 2tq+1), (page 16w+g+8, heads 2tq, 2tq+1)
    const int p0 = (blk0 + i) * kQmPages;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int pg = p0 + warp * 16 + g + (e >> 1) * 8;
      const int hh = chunk * 8 + 2 * tq + (e & 1);
      if (pg < p.np && hh < p.G) {
        const float v = pg >= p.force_from ? INFINITY : acc[e] * p.scaling;
        p.bounds[(int64_t(b) * p.Hq + hk * p.G + hh) * p.np + pg] = v;
      }
    }
  }
}

__global__ void quest_expand_kernel(const int64_t* pidx, int npick, int page, int S, int rows, void* out, int out64,
                                    int64_t o_rs) {
  griddep_wait();  // programmatic launch: the previous kernel's results are complete past here
  griddep_launch_dependents();
  const int row = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= npick * page || row >= rows) return;
  const int64_t pg = pidx[int64_t(row) * npick + i / page];
  int64_t t = pg * page + i % page;
  if (t > int64_t(S) - 1) t = int64_t(S) - 1;
  if (out64) reinterpret_cast<int64_t*>(out)[int64_t(row) * o_rs + i] = t;
  else reinterpret_cast<int32_t*>(out)[int64_t(row) * o_rs + i] = int32_t(t);
}

int run_topk(const float* scores, int rows, int rows_per_b, int64_t b_stride, int64_t row_stride, int n, int k,
             float* vals, int64_t v_rs, void* idx, int idx64, int64_t i_rs, int sorted, cudaStream_t st) {
  TopkParams p{};
  p.scores = scores; p.row_stride = row_stride; p.rows_per_b = rows_per_b; p.b_stride = b_stride;
  p.n = n; p.k = k; p.vals = vals; p.v_rs = v_rs; p.idx = idx; p.i_rs = i_rs; p.idx64 = idx64; p.sorted = sorted;
  const int kk = std::min(k, n);
  size_t wbytes = 0;
  if (sorted) {
    int kp = 1;
    while (kp < std::max(kk, 1)) kp <<= 1;
    wbytes = size_t(kp) * 8;
  }
  const bool in_smem = n <= kSmemRowMax;
  const size_t smem = (in_smem ? size_t(n) * 4 : 0) + wbytes;
  if (smem > 220 * 1024) return fail(BD_ERR_UNSUPPORTED, "top-k: sorted output of this many elements does not fit");
  int rc;
  if (n > 0 && n <= kSmRowMax && (!sorted || kk <= kSmSortMax)) {
    const size_t sm = sorted ? wbytes : 0;
    auto kern = n <= kSmThreads * 4 ? topk_small_kernel<4> : n <= kSmThreads * 8 ? topk_small_kernel<8>
                                                                                 : topk_small_kernel<16>;
    return launch_programmatic(kern, dim3(rows), dim3(kSmThreads), sm, st, p, "topk_small_kernel launch");
  }
  const size_t fast_smem = size_t(n) * 4 + 4096 * 4 + size_t(kCandMax) * 4 + wbytes;
  const bool aligned = (reinterpret_cast<uintptr_t>(scores) & 15) == 0 && row_stride % 4 == 0 &&
                       (rows_per_b >= rows || b_stride % 4 == 0);
  if (in_smem && n % 4 == 0 && n > 0 && aligned && fast_smem <= 220 * 1024) {
    static bool attr_f[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_f[dev & 63]) {
      if ((rc = cuda_check(cudaFuncSetAttribute(topk_fast_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                220 * 1024),
                           "cudaFuncSetAttribute(topk_fast)")))
        return rc;
      attr_f[dev & 63] = true;
    }
    // a plain launch: launched early behind the score pass, these one-per-SM CTAs measured
    // 20 us slower at c3's shape
    topk_fast_kernel<<<rows, kTkThreads, fast_smem, st>>>(p);
    return cuda_check(cudaGetLastError(), "topk_fast_kernel launch");
  }
  if (in_smem) {
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
      if ((rc = cuda_check(cudaFuncSetAttribute(topk_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024),
                           "cudaFuncSetAttribute(topk)")))
        return rc;
      attr[dev & 63] = true;
    }
    topk_kernel<true><<<rows, kTkThreads, smem, st>>>(p);
  } else {
    static bool attr2[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr2[dev & 63]) {
      if ((rc = cuda_check(cudaFuncSetAttribute(topk_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024),
                           "cudaFuncSetAttribute(topk)")))
        return rc;
      attr2[dev & 63] = true;
    }
    topk_kernel<false><<<rows, kTkThreads, smem, st>>>(p);
  }
  return cuda_check(cudaGetLastError(), "topk_kernel launch");
}

}  // namespace

// Index-list splits of the gather-attention: enough 4-warp CTAs for about two per SM, at
// least 64 index entries per split. Longer runs per CTA beat more splits (measured at c3:
// one split per row, 512 CTAs, then no combine at all).
int gather_splits(int64_t rows, int64_t kb) {
  const int64_t target = 2LL * num_sms();
  const int64_t want = std::max<int64_t>(1, (target + std::max<int64_t>(rows, 1) - 1) / std::max<int64_t>(rows, 1));
  return int(std::max<int64_t>(1, std::min<int64_t>(want, (kb + 63) / 64)));
}

}  // namespace bd

extern "C" {

int bd_topk(const bd_tensor* scores, int k, int sorted, const bd_tensor* values, const bd_tensor* indices,
            bd_stream_t stream) {
  using namespace bd;
  int rc;
  if (!scores) return fail(BD_ERR_NULL, "scores is NULL");
  const int nd = scores->ndim;
  if (nd < 1 || nd > 3) return fail(BD_ERR_SHAPE, "scores must have 1 to 3 dims");
  if ((rc = check_tensor(scores, "scores", nd, BD_F32)) || (rc = check_tensor(indices, "indices", nd))) return rc;
  if (indices->dtype != BD_I64 && indices->dtype != BD_I32) return fail(BD_ERR_DTYPE, "indices must be int64 or int32");
  if (values && (rc = check_tensor(values, "values", nd, BD_F32))) return rc;
  const int64_t n = scores->shape[nd - 1];
  if (k < 0) return fail(BD_ERR_VALUE, "k must be >= 0");
  if (k > n) return fail(BD_ERR_VALUE, "selected index k out of range");
  if (n > INT32_MAX / 2) return fail(BD_ERR_UNSUPPORTED, "row too long");
  int64_t rows = 1;
  for (int i = 0; i + 1 < nd; ++i) {
    rows *= scores->shape[i];
    if (indices->shape[i] != scores->shape[i] || (values && values->shape[i] != scores->shape[i]))
      return fail(BD_ERR_SHAPE, "leading dims of outputs must match scores");
  }
  if (indices->shape[nd - 1] != k || (values && values->shape[nd - 1] != k))
    return fail(BD_ERR_SHAPE, "outputs must have k in the last dim");
  if (scores->stride[nd - 1] != 1 && n > 1) return fail(BD_ERR_STRIDE, "scores rows must be contiguous");
  // rows addressed as (outer, inner) over at most two leading dims
  int64_t rows_per_b = nd == 3 ? scores->shape[1] : (nd == 2 ? scores->shape[0] : 1);
  int64_t row_stride = nd >= 2 ? scores->stride[nd - 2] : 0;
  int64_t b_stride = nd == 3 ? scores->stride[0] : 0;
  auto dense_rows = [&](const bd_tensor* t) {
    if (t->stride[nd - 1] != 1 && k > 1) return false;
    int64_t s = k;
    for (int i = nd - 2; i >= 0; --i) {
      if (t->shape[i] > 1 && t->stride[i] != s) return false;
      s *= t->shape[i];
    }
    return true;
  };
  if (!dense_rows(indices) || (values && !dense_rows(values))) return fail(BD_ERR_STRIDE, "outputs must be contiguous");
  if (rows == 0 || k == 0) return BD_OK;
  if (rows > INT32_MAX) return fail(BD_ERR_UNSUPPORTED, "too many rows");
  return run_topk(static_cast<const float*>(scores->data), int(rows), int(rows_per_b), b_stride, row_stride, int(n), k,
                  values ? static_cast<float*>(values->data) : nullptr, k, indices->data, indices->dtype == BD_I64, k,
                  sorted, reinterpret_cast<cudaStream_t>(stream));
}

size_t bd_sparse_gather_attn_workspace(const bd_tensor* q, const bd_tensor* idx) {
  using namespace bd;
  if (check_tensor(q, "q", 3) || check_tensor(idx, "idx", 3)) return 0;
  const int64_t rows = q->shape[0] * q->shape[1];
  return partials_bytes(size_t(rows), gather_splits(rows, idx->shape[2]), int(q->shape[2]));
}

// Gather-attend over idx into split partials, then either the final output (`out`) or one
// exported (m, l, o) per row (`em`, `el`, `eo`: the shard partial of a multi-GPU exchange).
static int sparse_gather_run(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v, const bd_tensor* idx,
                             float scaling, const bd_tensor* out, const bd_tensor* em, const bd_tensor* el,
                             const bd_tensor* eo, void* workspace, size_t workspace_bytes, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if ((rc = check_tensor(q, "q", 3)) || (rc = check_tensor(k, "k", 4)) || (rc = check_tensor(v, "v", 4)) ||
      (rc = check_tensor(idx, "idx", 3)))
    return rc;
  if (out ? (rc = check_tensor(out, "out", 3))
          : ((rc = check_tensor(em, "m", 2, BD_F32)) || (rc = check_tensor(el, "l", 2, BD_F32)) ||
             (rc = check_tensor(eo, "o", 3, BD_F32))))
    return rc;
  if (k->dtype != v->dtype ||
      (k->dtype != BD_BF16 && k->dtype != BD_F8E4M3 && k->dtype != BD_F16 && k->dtype != BD_F32))
    return fail(BD_ERR_DTYPE, "k and v must share one dtype: bf16, fp8 e4m3, f16 or f32");
  if (idx->dtype != BD_I32 && idx->dtype != BD_I64) return fail(BD_ERR_DTYPE, "idx must be int32 or int64");
  if (q->dtype != BD_BF16 && q->dtype != BD_F16 && q->dtype != BD_F32) return fail(BD_ERR_DTYPE, "q must be bf16/f16/f32");
  const int64_t B = q->shape[0], Hq = q->shape[1], D = q->shape[2];
  const int64_t Hk = k->shape[1], S = k->shape[2], kb = idx->shape[2];
  if (Hk <= 0 || Hq % Hk) return fail(BD_ERR_SHAPE, "H_q must be a multiple of H_k");
  if (D != 32 && D != 64 && D != 128) return fail(BD_ERR_UNSUPPORTED, "head_dim must be 32, 64 or 128");
  for (int i = 0; i < 4; ++i)
    if (k->shape[i] != v->shape[i]) return fail(BD_ERR_SHAPE, "k and v shapes differ");
  if (k->shape[0] != B || k->shape[3] != D || idx->shape[0] != B || idx->shape[1] != Hq)
    return fail(BD_ERR_SHAPE, "expect q [B,Hq,D], k/v [B,Hk,S,D], idx [B,Hq,kb]");
  if (out && (out->shape[0] != B || out->shape[1] != Hq || out->shape[2] != D || out->stride[2] != 1))
    return fail(BD_ERR_SHAPE, "out must be [B,Hq,D] with contiguous rows");
  if (!out) {
    if (em->shape[0] != B || em->shape[1] != Hq || el->shape[0] != B || el->shape[1] != Hq || eo->shape[0] != B ||
        eo->shape[1] != Hq || eo->shape[2] != D)
      return fail(BD_ERR_SHAPE, "m,l must be [B,Hq] and o [B,Hq,D]");
    if (em->stride[1] != 1 || em->stride[0] != Hq || el->stride[1] != 1 || el->stride[0] != Hq ||
        eo->stride[2] != 1 || eo->stride[1] != D || eo->stride[0] != Hq * D)
      return fail(BD_ERR_STRIDE, "m, l, o must be contiguous");
  }
  if (idx->stride[2] != 1 && kb > 1) return fail(BD_ERR_STRIDE, "idx rows must be contiguous");
  if (q->stride[2] != 1) return fail(BD_ERR_STRIDE, "q innermost dim must be contiguous");
  if ((rc = check_rows_aligned(k, "k")) || (rc = check_rows_aligned(v, "v"))) return rc;
  if (B * Hq == 0) return BD_OK;
  const int64_t rows = B * Hq;
  const int nsplit = gather_splits(rows, kb);
  const size_t need = partials_bytes(size_t(rows), nsplit, int(D));
  if (!workspace || workspace_bytes < need) return fail(BD_ERR_WORKSPACE, "need " + std::to_string(need) + " workspace bytes");
  Partials part = carve_partials(workspace, size_t(rows), nsplit, int(D));
  GatherParams p{};
  p.q = q->data; p.q_sb = q->stride[0]; p.q_sh = q->stride[1]; p.q_dtype = q->dtype;
  p.k = static_cast<const uint8_t*>(k->data); p.k_sb = k->stride[0]; p.k_sh = k->stride[1]; p.k_ss = k->stride[2];
  p.v = static_cast<const uint8_t*>(v->data); p.v_sb = v->stride[0]; p.v_sh = v->stride[1]; p.v_ss = v->stride[2];
  p.idx = idx->data; p.i_sb = idx->stride[0]; p.i_sh = idx->stride[1]; p.idx64 = idx->dtype == BD_I64;
  p.B = int(B); p.Hq = int(Hq); p.Hk = int(Hk); p.G = int(Hq / Hk); p.S = int(S); p.kb = int(kb);
  p.scaling = scaling;
  p.rows_per_split = int((kb + nsplit - 1) / nsplit);
  p.nsplit = nsplit;
  p.part_m = part.m; p.part_l = part.l; p.part_o = part.o;
  const bool direct = nsplit == 1;
  if (direct && out) {
    p.out = out->data; p.out_dtype = out->dtype; p.o_sb = out->stride[0]; p.o_sh = out->stride[1];
  } else if (direct) {  // the row's (m, l, o) are the exported partial
    p.part_m = static_cast<float*>(em->data); p.part_l = static_cast<float*>(el->data);
    p.part_o = static_cast<float*>(eo->data);
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  dim3 grid(nsplit, unsigned(Hq), unsigned(B));
  const int kv = k->dtype == BD_F8E4M3 ? kGvFp8 : k->dtype == BD_F16 ? kGvF16 : k->dtype == BD_F32 ? kGvF32 : kGvBf16;
  auto pick = [&](auto d) {
    constexpr int DD = decltype(d)::value;
    return kv == kGvFp8 ? gather_attn_kernel<DD, kGvFp8>
         : kv == kGvF16 ? gather_attn_kernel<DD, kGvF16>
         : kv == kGvF32 ? gather_attn_kernel<DD, kGvF32> : gather_attn_kernel<DD, kGvBf16>;
  };
  auto kern = D == 128 ? pick(std::integral_constant<int, 128>{})
            : D == 64 ? pick(std::integral_constant<int, 64>{}) : pick(std::integral_constant<int, 32>{});
  rc = launch_programmatic(kern, grid, dim3(128), 0, st, p, "gather_attn_kernel launch");
  if (rc) return rc;
  if (direct) return BD_OK;
  if (out) return launch_combine(part, int(B), int(Hq), int(D), out, st, true);
  return launch_combine_export(part, int(B), int(Hq), int(D), static_cast<float*>(em->data),
                               static_cast<float*>(el->data), static_cast<float*>(eo->data), st, true);
}


int bd_sparse_gather_attn(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v, const bd_tensor* idx,
                          float scaling, const bd_tensor* out, void* workspace, size_t workspace_bytes,
                          bd_stream_t stream) {
  if (!out) return bd::fail(BD_ERR_NULL, "out is NULL");
  return sparse_gather_run(q, k, v, idx, scaling, out, nullptr, nullptr, nullptr, workspace, workspace_bytes, stream);
}

int bd_sparse_gather_attn_partial(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v, const bd_tensor* idx,
                                  float scaling, const bd_tensor* m, const bd_tensor* l, const bd_tensor* o,
                                  void* workspace, size_t workspace_bytes, bd_stream_t stream) {
  if (!m || !l || !o) return bd::fail(BD_ERR_NULL, "m, l or o is NULL");
  return sparse_gather_run(q, k, v, idx, scaling, nullptr, m, l, o, workspace, workspace_bytes, stream);
}

int bd_quest_page_minmax(const bd_tensor* k, int page, const bd_tensor* kmin, const bd_tensor* kmax,
                         bd_stream_t stream) {
  using namespace bd;
  int rc;
  if ((rc = check_tensor(k, "k", 4)) || (rc = check_tensor(kmin, "kmin", 4, k->dtype)) ||
      (rc = check_tensor(kmax, "kmax", 4, k->dtype)))
    return rc;
  if (page <= 0) return fail(BD_ERR_VALUE, "page must be positive");
  if (k->dtype != BD_BF16 && k->dtype != BD_F16 && k->dtype != BD_F32) return fail(BD_ERR_DTYPE, "k must be bf16/f16/f32");
  const int64_t B = k->shape[0], H = k->shape[1], S = k->shape[2], D = k->shape[3];
  const int64_t np = (S + page - 1) / page;
  for (int i = 0; i < 4; ++i)
    if (kmin->stride[i] != kmax->stride[i]) return fail(BD_ERR_STRIDE, "kmin and kmax must share a layout");
  for (const bd_tensor* t : {kmin, kmax}) {
    if (t->shape[0] != B || t->shape[1] != H || t->shape[2] != np || t->shape[3] != D)
      return fail(BD_ERR_SHAPE, "kmin/kmax must be [B,H,ceil(S/page),D]");
    if (D > 1 && t->stride[3] != 1) return fail(BD_ERR_STRIDE, "kmin/kmax channels must be contiguous");
  }
  if (B * H * np * D == 0) return BD_OK;
  const int64_t per_b = H * np * D;
  dim3 grid(unsigned((per_b + 255) / 256), unsigned(B));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (k->dtype == BD_BF16)
    quest_minmax_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(k->data), k->stride[0],
        k->stride[1], k->stride[2], int(H), int(S), int(D), page, int(np), static_cast<__nv_bfloat16*>(kmin->data),
        static_cast<__nv_bfloat16*>(kmax->data), kmin->stride[0], kmin->stride[1], kmin->stride[2]);
  else if (k->dtype == BD_F16)
    quest_minmax_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(k->data), k->stride[0], k->stride[1],
        k->stride[2], int(H), int(S), int(D), page, int(np), static_cast<__half*>(kmin->data),
        static_cast<__half*>(kmax->data), kmin->stride[0], kmin->stride[1], kmin->stride[2]);
  else
    quest_minmax_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(k->data), k->stride[0], k->stride[1],
        k->stride[2], int(H), int(S), int(D), page, int(np), static_cast<float*>(kmin->data),
        static_cast<float*>(kmax->data), kmin->stride[0], kmin->stride[1], kmin->stride[2]);
  return cuda_check(cudaGetLastError(), "quest_minmax_kernel launch");
}

int bd_quest_page_bounds(const bd_tensor* q, const bd_tensor* kmin, const bd_tensor* kmax, float scaling,
                         int force_from_page, const bd_tensor* bounds, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if ((rc = check_tensor(q, "q", 3)) || (rc = check_tensor(kmin, "kmin", 4)) ||
      (rc = check_tensor(kmax, "kmax", 4, kmin->dtype)) || (rc = check_tensor(bounds, "bounds", 3, BD_F32)))
    return rc;
  if (kmin->dtype != BD_BF16 && kmin->dtype != BD_F16 && kmin->dtype != BD_F32)
    return fail(BD_ERR_DTYPE, "kmin/kmax must be bf16, f16 or f32");
  if (q->dtype != BD_BF16 && q->dtype != BD_F16 && q->dtype != BD_F32) return fail(BD_ERR_DTYPE, "q must be bf16/f16/f32");
  const int64_t B = q->shape[0], Hq = q->shape[1], D = q->shape[2];
  const int64_t Hk = kmin->shape[1], np = kmin->shape[2];
  if (Hk <= 0 || Hq % Hk) return fail(BD_ERR_SHAPE, "H_q must be a multiple of H_k");
  if (D != 32 && D != 64 && D != 128) return fail(BD_ERR_UNSUPPORTED, "head_dim must be 32, 64 or 128");
  for (int i = 0; i < 4; ++i)
    if (kmin->shape[i] != kmax->shape[i] || kmin->stride[i] != kmax->stride[i])
      return fail(BD_ERR_SHAPE, "kmin and kmax must have the same shape and layout");
  if (kmin->shape[0] != B || kmin->shape[3] != D) return fail(BD_ERR_SHAPE, "kmin must be [B,Hk,np,D]");
  if (bounds->shape[0] != B || bounds->shape[1] != Hq || bounds->shape[2] != np || bounds->stride[2] != 1 ||
      bounds->stride[1] != np || (B > 1 && bounds->stride[0] != Hq * np))
    return fail(BD_ERR_SHAPE, "bounds must be contiguous [B,Hq,np]");
  if (q->stride[2] != 1) return fail(BD_ERR_STRIDE, "q innermost dim must be contiguous");
  if ((rc = check_rows_aligned(kmin, "kmin")) || (rc = check_rows_aligned(kmax, "kmax"))) return rc;
  if (B * Hq * np == 0) return BD_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  auto* mn = static_cast<const __nv_bfloat16*>(kmin->data);
  auto* mx = static_cast<const __nv_bfloat16*>(kmax->data);
  // bf16 query and metadata with 4-byte aligned channel pairs: tensor-core bounds (bf16
  // products are exact in fp32)
  if (kmin->dtype == BD_BF16 && q->dtype == BD_BF16 && (reinterpret_cast<uintptr_t>(q->data) & 3) == 0 &&
      (q->stride[0] % 2) == 0 && (q->stride[1] % 2) == 0) {
    QuestMmaParams p{};
    p.q = static_cast<const __nv_bfloat16*>(q->data); p.q_sb = q->stride[0]; p.q_sh = q->stride[1];
    p.kmin = mn; p.kmax = mx; p.m_sb = kmin->stride[0]; p.m_sh = kmin->stride[1]; p.m_sp = kmin->stride[2];
    p.Hq = int(Hq); p.Hk = int(Hk); p.G = int(Hq / Hk); p.head_chunks = (p.G + 7) / 8; p.np = int(np);
    p.force_from = force_from_page; p.scaling = scaling; p.bounds = static_cast<float*>(bounds->data);
    // enough CTAs for one wave at three per SM; each streams an equal run of page blocks
    const int64_t nblk = (np + kQmPages - 1) / kQmPages;
    const int64_t groups = int64_t(B) * Hk * p.head_chunks;
    const int64_t per_group = std::max<int64_t>(1, std::min<int64_t>(nblk, 3LL * num_sms() / std::max<int64_t>(groups, 1)));
    p.blocks_per_cta = int((nblk + per_group - 1) / per_group);
    dim3 gm(unsigned((nblk + p.blocks_per_cta - 1) / p.blocks_per_cta), unsigned(Hk * p.head_chunks), unsigned(B));
    const size_t smem = size_t(2) * kQmPages * (4 * D + 16);
    auto launch = [&](auto kern) {
      // one flag per head_dim instance and device: the instances need different sizes
      static bool attr[3][64] = {};
      const int di = D == 128 ? 2 : D == 64 ? 1 : 0;
      int dev = 0;
      cudaGetDevice(&dev);
      if (!attr[di][dev & 63]) {
        const int r = cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
                                 "cudaFuncSetAttribute(quest_bounds)");
        if (r) return r;
        attr[di][dev & 63] = true;
      }
      return launch_programmatic(kern, gm, dim3(128), smem, st, p, "quest_bounds_mma_kernel launch");
    };
    if (D == 128) return launch(quest_bounds_mma_kernel<128>);
    if (D == 64) return launch(quest_bounds_mma_kernel<64>);
    return launch(quest_bounds_mma_kernel<32>);
  }
  auto run = [&](auto tag) {
    using MT = decltype(tag);
    constexpr int NP = sizeof(MT) == 4 ? kQPages / 2 : kQPages;
    dim3 grid(unsigned((np + NP - 1) / NP), unsigned(Hk), unsigned(B));
    auto kern = D == 128 ? quest_bounds_kernel<128, MT> : D == 64 ? quest_bounds_kernel<64, MT> : quest_bounds_kernel<32, MT>;
    return launch_pdl(kern, grid, dim3(NP), 0, st, "quest_bounds_kernel launch", q->data, q->dtype, q->stride[0],
                      q->stride[1], static_cast<const MT*>(kmin->data), static_cast<const MT*>(kmax->data),
                      kmin->stride[0], kmin->stride[1], kmin->stride[2], int(Hq), int(Hk), int(np), scaling,
                      force_from_page, static_cast<float*>(bounds->data));
  };
  if (kmin->dtype == BD_F32) return run(float{});
  if (kmin->dtype == BD_F16) return run(__half{});
  return run(__nv_bfloat16{});
}

size_t bd_quest_select_workspace(const bd_tensor* q, const bd_tensor* kmin, int kb, int page) {
  using namespace bd;
  if (check_tensor(q, "q", 3) || check_tensor(kmin, "kmin", 4) || page <= 0) return 0;
  const int64_t np = kmin->shape[2];
  const int64_t npick = std::min<int64_t>(std::max<int64_t>(1, (kb + page - 1) / page), np);
  const int64_t rows = q->shape[0] * q->shape[1];
  return size_t(rows * np * 4 + rows * npick * 8 + 512);
}

int bd_quest_select(const bd_tensor* q, const bd_tensor* kmin, const bd_tensor* kmax, int S, int kb, int page,
                    float scaling, int force_from_page, const bd_tensor* idx_out, void* workspace,
                    size_t workspace_bytes, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if ((rc = check_tensor(q, "q", 3)) || (rc = check_tensor(kmin, "kmin", 4)) || (rc = check_tensor(idx_out, "idx", 3)))
    return rc;
  if (page <= 0 || kb < 0 || S <= 0) return fail(BD_ERR_VALUE, "page, kb and S must be positive");
  const int64_t B = q->shape[0], Hq = q->shape[1];
  const int64_t np = kmin->shape[2];
  if (np != (S + page - 1) / page) return fail(BD_ERR_SHAPE, "page metadata does not match S and page");
  const int64_t npick = std::min<int64_t>(std::max<int64_t>(1, (kb + page - 1) / page), np);
  if (idx_out->dtype != BD_I32 && idx_out->dtype != BD_I64) return fail(BD_ERR_DTYPE, "idx must be int32 or int64");
  if (idx_out->shape[0] != B || idx_out->shape[1] != Hq || idx_out->shape[2] != npick * page || idx_out->stride[2] != 1 ||
      idx_out->stride[1] != npick * page || (B > 1 && idx_out->stride[0] != Hq * npick * page))
    return fail(BD_ERR_SHAPE, "idx must be contiguous [B,Hq,npick*page]");
  const int64_t rows = B * Hq;
  const size_t need = size_t(rows * np * 4 + rows * npick * 8 + 512);
  if (!workspace || workspace_bytes < need) return fail(BD_ERR_WORKSPACE, "need " + std::to_string(need) + " workspace bytes");
  if (rows == 0) return BD_OK;
  uintptr_t base = (reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255);
  float* bounds = reinterpret_cast<float*>(base);
  int64_t* pidx = reinterpret_cast<int64_t*>((base + size_t(rows * np * 4) + 255) & ~uintptr_t(255));
  bd_tensor bt{};
  bt.data = bounds; bt.dtype = BD_F32; bt.ndim = 3;
  bt.shape[0] = B; bt.shape[1] = Hq; bt.shape[2] = np;
  bt.stride[0] = Hq * np; bt.stride[1] = np; bt.stride[2] = 1;
  if ((rc = bd_quest_page_bounds(q, kmin, kmax, scaling, force_from_page, &bt, stream))) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if ((rc = run_topk(bounds, int(rows), int(rows), 0, np, int(np), int(npick), nullptr, 0, pidx, 1, npick, 1, st)))
    return rc;
  dim3 grid(unsigned((npick * page + 255) / 256), unsigned(rows));
  return launch_pdl(quest_expand_kernel, grid, dim3(256), 0, st, "quest_expand_kernel launch",
                    static_cast<const int64_t*>(pidx), int(npick), page, S, int(rows), idx_out->data,
                    int(idx_out->dtype == BD_I64), int64_t(npick * page));
}

}  // extern "C"
