// Split-KV across GPUs over NVLink peer memory: the merge of this rank's split partials,
// the all-gather of the per-rank (max, sum, numerator) and their log-sum-exp combine in one
// kernel, launched right behind the dense split pass over this rank's token shard.
//
// Every rank owns one buffer that all ranks can address (a symmetric allocation mapped on
// every GPU of the NVSwitch domain), zero before the first call:
//   records   f32 [2 parities][world][rows][D + 4]   o[D], m, l, 0, 0   (16-byte aligned rows)
//   flags     u32 [2 parities][world][rows]
//   counters  u32 [rows]                              steps done, read only by the owner
// The grid has at most one CTA per SM; CTA c owns rows c, c + grid, ... (row = b*Hq + hq).
// Step s = counter + 1 uses parity s & 1. For each of its rows the CTA merges the row's n
// source partials (n = 1 for partials the caller computed) and stores the merged record into
// slot [parity][rank][row] of every rank's buffer (plain peer stores); it then fences at
// system scope, writes s into flag [parity][rank][row] of every rank with release semantics,
// waits, with acquire loads and a time limit, until flags [parity][*][row] of its own buffer
// read s for all its rows, combines the world records into `out` and stores s into the
// rows' counters. All CTAs are resident together and publish before they wait, so no wait
// depends on a CTA that has not been scheduled.
// The counter lives in device memory, so a captured call can be replayed from a CUDA graph.
// Two parities are enough: rank r can only write step s + 2 of a row after every rank has
// raised that row's flag for step s + 1, which each does only in a launch that starts after
// its own step-s launch (and its reads of step s's records) has finished.
//
// The reference is single-GPU and has no counterpart; the merge is the online-softmax
// identity its kernels apply across key blocks (src/attention_kernels.py:45-59 of
// saifmb0/bytes).
#include "decode_shared.cuh"

namespace bd {
namespace {

constexpr int kExThreads = 256;
constexpr int kMaxWorld = 64;
// ranks are separate processes whose launches may be skewed by host-side pauses, so the wait
// for the peers' flags gets a longer limit than the in-kernel tile waits
constexpr uint64_t kPeerWaitNs = 1000ull * 1000ull * 1000ull;  // 1 s

// waits that ran past their limit (the combined output of that call is NaN)
__device__ unsigned int g_exchange_timeouts = 0;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct ExchangeParams {
  // this rank's source partials of row r: m,l at r*n + i, o at (r*n + i)*D, i < n
  const float* m; const float* l; const float* o;
  int n;
  float* const* peers;  // device array [world] of buffer bases
  int rank, world, rows, D, Hq;
  void* out; int out_dtype; int64_t o_sb, o_sh;
};

__host__ __device__ inline int64_t record_floats(int D) { return int64_t(D) + 4; }
__host__ __device__ inline int64_t flags_offset(int rows, int D, int world) {  // in floats
  return 2 * int64_t(world) * rows * record_floats(D);
}

__global__ void __launch_bounds__(kExThreads) peer_exchange_kernel(const ExchangeParams p) {
  griddep_wait();  // the split pass of a programmatic predecessor (no-op after a plain launch)
  const int tid = threadIdx.x;
  const int D4 = p.D / 4, rec4 = D4 + 1;
  const int64_t rec = record_floats(p.D);
  float* own = p.peers[p.rank];
  uint32_t* own_flags = reinterpret_cast<uint32_t*>(own + flags_offset(p.rows, p.D, p.world));
  uint32_t* counters = own_flags + 2 * int64_t(p.world) * p.rows;
  // every row of one call advances together; the first row of this CTA gives the step
  const uint32_t step = counters[blockIdx.x] + 1u;
  const int par = int(step & 1u);
  auto slot_of = [&](int r, int row) { return (int64_t(par) * p.world + r) * p.rows + row; };

  extern __shared__ __align__(16) float sm[];
  float4* rec_s = reinterpret_cast<float4*>(sm);      // [rec4] the merged record
  float* red = sm + 4 * rec4;                          // [ns][D] slice sums
  const int ns = kExThreads / D4;
  float* wts = red + ns * p.D;                         // [n] split weights
  __shared__ float sM, sL, rm[kMaxWorld], rl[kMaxWorld];

  // ---- 1. per row of this CTA: merge its n source partials into one record (o un-normalised,
  // m, l) and store it into slot [par][rank][row] of every rank's buffer
  for (int row = blockIdx.x; row < p.rows; row += gridDim.x) {
    if (tid < 32) {
      float M = -INFINITY;
      for (int i = tid; i < p.n; i += 32) M = fmaxf(M, p.m[int64_t(row) * p.n + i]);
      M = warp_max(M);
      float L = 0.f;
      for (int i = tid; i < p.n; i += 32) {
        const float w = M == -INFINITY ? 0.f : __expf(p.m[int64_t(row) * p.n + i] - M);
        wts[i] = w;
        L = fmaf(p.l[int64_t(row) * p.n + i], w, L);
      }
      L = warp_sum(L);
      if (tid == 0) { sM = M; sL = L; }
    }
    __syncthreads();
    {
      const int ci = tid % D4, sl = tid / D4;
      if (sl < ns) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        const float4* src = reinterpret_cast<const float4*>(p.o + int64_t(row) * p.n * p.D) + ci;
#pragma unroll 4
        for (int i = sl; i < p.n; i += ns) {
          const float4 v = src[int64_t(i) * D4];
          const float w = wts[i];
          acc.x = fmaf(v.x, w, acc.x); acc.y = fmaf(v.y, w, acc.y);
          acc.z = fmaf(v.z, w, acc.z); acc.w = fmaf(v.w, w, acc.w);
        }
        reinterpret_cast<float4*>(red)[sl * D4 + ci] = acc;
      }
    }
    __syncthreads();
    if (tid < D4) {
      float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int s = 0; s < ns; ++s) {
        const float4 v = reinterpret_cast<const float4*>(red)[s * D4 + tid];
        O.x += v.x; O.y += v.y; O.z += v.z; O.w += v.w;
      }
      rec_s[tid] = O;
    } else if (tid == D4) {
      rec_s[D4] = make_float4(sM, sL, 0.f, 0.f);
    }
    __syncthreads();
    for (int i = tid; i < p.world * rec4; i += kExThreads) {
      const int r = i / rec4, j = i - r * rec4;
      reinterpret_cast<float4*>(p.peers[r] + slot_of(p.rank, row) * rec)[j] = rec_s[j];
    }
    __syncthreads();  // rec_s and wts are reused by the next row
  }

  // ---- 2. every thread's peer stores are visible system-wide before any flag is raised;
  // then flag [par][rank][row] of every rank, for each row of this CTA
  __threadfence_system();
  __syncthreads();
  const int mine = (p.rows - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x);
  for (int i = tid; i < mine * p.world; i += kExThreads) {
    const int row = int(blockIdx.x) + (i / p.world) * int(gridDim.x), r = i % p.world;
    uint32_t* flags = reinterpret_cast<uint32_t*>(p.peers[r] + flags_offset(p.rows, p.D, p.world));
    st_release_sys(flags + slot_of(p.rank, row), step);
  }

  // ---- 3. wait for every rank's flags of this CTA's rows in this rank's own buffer (bounded)
  bool late = false;
  for (int i = tid; i < mine * p.world; i += kExThreads) {
    const int row = int(blockIdx.x) + (i / p.world) * int(gridDim.x), r = i % p.world;
    const uint32_t* f = own_flags + slot_of(r, row);
    if (ld_acquire_sys(f) != step) {
      const uint64_t t0 = globaltimer_ns();
      for (;;) {
        if (ld_acquire_sys(f) == step) break;
        if (globaltimer_ns() - t0 > kPeerWaitNs) {
          late = true;
          break;
        }
      }
    }
  }
  const bool failed = __syncthreads_or(late);
  if (failed && tid == 0) atomicAdd(&g_exchange_timeouts, 1u);

  // ---- 4. combine each row: out[c] = sum_r o_r[c] e^(m_r - M) / sum_r l_r e^(m_r - M)
  for (int row = blockIdx.x; row < p.rows; row += gridDim.x) {
    if (tid < p.world) {
      const float4 ml = reinterpret_cast<const float4*>(own + slot_of(tid, row) * rec)[D4];
      rm[tid] = ml.x;
      rl[tid] = ml.y;
    }
    __syncthreads();
    if (tid < D4) {
      float M = -INFINITY;
      for (int r = 0; r < p.world; ++r) M = fmaxf(M, rm[r]);
      float L = 0.f;
      float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < p.world; ++r) {
        const float w = M == -INFINITY ? 0.f : __expf(rm[r] - M);
        L = fmaf(rl[r], w, L);
        const float4 v = reinterpret_cast<const float4*>(own + slot_of(r, row) * rec)[tid];
        O.x = fmaf(v.x, w, O.x); O.y = fmaf(v.y, w, O.y); O.z = fmaf(v.z, w, O.z); O.w = fmaf(v.w, w, O.w);
      }
      const float inv = 1.f / L;
      const float nan = __int_as_float(0x7fc00000);
      const int64_t off = int64_t(row / p.Hq) * p.o_sb + int64_t(row % p.Hq) * p.o_sh + 4 * tid;
      store_as(p.out, p.out_dtype, off, failed ? nan : O.x * inv);
      store_as(p.out, p.out_dtype, off + 1, failed ? nan : O.y * inv);
      store_as(p.out, p.out_dtype, off + 2, failed ? nan : O.z * inv);
      store_as(p.out, p.out_dtype, off + 3, failed ? nan : O.w * inv);
    }
    __syncthreads();  // rm, rl are reused by the next row
  }
  // every thread read the step before the first barrier
  for (int row = int(blockIdx.x) + tid * int(gridDim.x); row < p.rows; row += kExThreads * int(gridDim.x))
    counters[row] = step;
}

int check_out(const bd_tensor* out, int64_t B, int64_t Hq, int64_t D) {
  int rc;
  if ((rc = check_tensor(out, "out", 3))) return rc;
  if (out->shape[0] != B || out->shape[1] != Hq || out->shape[2] != D)
    return fail(BD_ERR_SHAPE, "out must be [B,Hq,D]");
  if (out->dtype != BD_BF16 && out->dtype != BD_F16 && out->dtype != BD_F32)
    return fail(BD_ERR_DTYPE, "out must be bf16, f16 or f32");
  if (out->stride[2] != 1) return fail(BD_ERR_STRIDE, "out innermost dim must be contiguous");
  return BD_OK;
}

int check_group(void* const* peer_buffers, int rank, int world, int64_t D) {
  if (!peer_buffers) return fail(BD_ERR_NULL, "peer_buffers is NULL");
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world)
    return fail(BD_ERR_VALUE, "need 1 <= world <= 64 and 0 <= rank < world");
  if (D <= 0 || D % 4 || D / 4 > kExThreads / 2)
    return fail(BD_ERR_UNSUPPORTED, "peer exchange needs head_dim a multiple of 4, at most 512");
  return BD_OK;
}

int launch_exchange(const ExchangeParams& p, cudaStream_t st, bool pdl) {
  if (p.rows == 0) return BD_OK;
  const int D4 = p.D / 4, ns = kExThreads / D4;
  const size_t smem = (size_t(4) * (D4 + 1) + size_t(ns) * p.D + size_t(p.n)) * sizeof(float);
  if (smem > 48 * 1024) return fail(BD_ERR_UNSUPPORTED, "peer exchange: too many split partials per row");
  // at most one CTA per SM, so every CTA of the grid is resident at once: each publishes all
  // of its rows before it waits on any, so no rank's wait depends on a CTA not yet scheduled
  const int grid = std::min(p.rows, num_sms());
  if (pdl)
    return launch_pdl(peer_exchange_kernel, dim3(grid), dim3(kExThreads), smem, st, "peer_exchange_kernel launch", p);
  peer_exchange_kernel<<<grid, kExThreads, smem, st>>>(p);
  return cuda_check(cudaGetLastError(), "peer_exchange_kernel launch");
}

}  // namespace

long long exchange_wait_timeouts() {
  unsigned int v = 0;
  return cudaMemcpyFromSymbol(&v, g_exchange_timeouts, sizeof v) == cudaSuccess ? (long long)v : -1;
}

}  // namespace bd

extern "C" {

size_t bd_peer_exchange_buffer_bytes(int rows, int D, int world) {
  using namespace bd;
  if (rows <= 0 || D <= 0 || world <= 0) return 0;
  const size_t floats = size_t(flags_offset(rows, D, world));
  const size_t words = 2 * size_t(world) * rows + size_t(rows);
  return ((floats + words) * 4 + 15) & ~size_t(15);
}

int bd_peer_exchange_combine(const bd_tensor* m, const bd_tensor* l, const bd_tensor* o, void* const* peer_buffers,
                             int rank, int world, const bd_tensor* out, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if ((rc = check_tensor(m, "m", 2, BD_F32)) || (rc = check_tensor(l, "l", 2, BD_F32)) ||
      (rc = check_tensor(o, "o", 3, BD_F32)))
    return rc;
  const int64_t B = m->shape[0], Hq = m->shape[1], D = o->shape[2];
  if (l->shape[0] != B || l->shape[1] != Hq || o->shape[0] != B || o->shape[1] != Hq)
    return fail(BD_ERR_SHAPE, "shapes must be m,l [B,Hq], o [B,Hq,D]");
  if ((rc = check_out(out, B, Hq, D)) || (rc = check_group(peer_buffers, rank, world, D))) return rc;
  if (m->stride[1] != 1 || m->stride[0] != Hq || l->stride[1] != 1 || l->stride[0] != Hq || o->stride[2] != 1 ||
      o->stride[1] != D || o->stride[0] != Hq * D)
    return fail(BD_ERR_STRIDE, "m, l, o must be contiguous");
  if (reinterpret_cast<uintptr_t>(o->data) & 15) return fail(BD_ERR_UNSUPPORTED, "o must be 16-byte aligned");
  ExchangeParams p{};
  p.m = static_cast<const float*>(m->data); p.l = static_cast<const float*>(l->data);
  p.o = static_cast<const float*>(o->data); p.n = 1;
  p.peers = reinterpret_cast<float* const*>(peer_buffers);
  p.rank = rank; p.world = world; p.rows = int(B * Hq); p.D = int(D); p.Hq = int(Hq);
  p.out = out->data; p.out_dtype = out->dtype; p.o_sb = out->stride[0]; p.o_sh = out->stride[1];
  return launch_exchange(p, reinterpret_cast<cudaStream_t>(stream), false);
}

int bd_split_kv_decode_peer(const bd_tensor* q, const bd_tensor* k, const bd_tensor* v, float scaling,
                            void* const* peer_buffers, int rank, int world, const bd_tensor* out, void* workspace,
                            size_t workspace_bytes, bd_stream_t stream) {
  using namespace bd;
  int rc;
  if ((rc = check_tensor(q, "q", 3)) || (rc = check_tensor(k, "k", 4))) return rc;
  const int64_t B = q->shape[0], Hq = q->shape[1], D = q->shape[2];
  if ((rc = check_out(out, B, Hq, D)) || (rc = check_group(peer_buffers, rank, world, D))) return rc;
  const int nsplit = dense_split_count(B, Hq, k->shape[1], k->shape[2], D, 0);
  if (nsplit <= 0) return fail(BD_ERR_SHAPE, "q and k shapes do not make a decode plan");
  const size_t rows = size_t(B) * size_t(Hq);
  if (rows == 0) return BD_OK;
  const size_t need = partials_bytes(rows, nsplit, int(D));
  if (!workspace || workspace_bytes < need)
    return fail(BD_ERR_WORKSPACE, "need " + std::to_string(need) + " workspace bytes");
  const Partials part = carve_partials(workspace, rows, nsplit, int(D));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if ((rc = launch_dense_partials(q, k, v, scaling, part, 0, nsplit, st, false))) return rc;
  ExchangeParams p{};
  p.m = part.m; p.l = part.l; p.o = part.o; p.n = nsplit;
  p.peers = reinterpret_cast<float* const*>(peer_buffers);
  p.rank = rank; p.world = world; p.rows = int(rows); p.D = int(D); p.Hq = int(Hq);
  p.out = out->data; p.out_dtype = out->dtype; p.o_sb = out->stride[0]; p.o_sh = out->stride[1];
  return launch_exchange(p, st, true);
}

}  // extern "C"
