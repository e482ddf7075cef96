// th_allreduce: in-place sum all-reduce of a byte range of a symmetric buffer
// through NVSwitch multicast (NVLS), one kernel per call on each rank.
//
// Every rank holds the same buffer layout, mapped three ways: its own
// (unicast) address, the peers' addresses of their copies (only their signal
// pads are touched that way) and one multicast address that reaches all
// copies.  Rank r owns slice r of the range (range / world bytes):
//
//   1. start barrier: block b stores `epoch` into block b's start slot of every
//      rank's signal pad (st.release.sys), then waits (bounded) until every
//      rank's block b has done the same -- so every rank's input rows (written
//      by kernels that precede this one on its stream) are complete;
//   2. multimem.ld_reduce over slice r: the switch reads the 16 bytes at that
//      address on every rank and returns their sum (fp32 accumulation for the
//      16-bit types); multimem.st writes the sum back to every rank's copy;
//   3. end barrier: the same handshake on the end slots, so no rank reuses the
//      buffer (or reads it) before every rank's stores into it have landed and
//      every rank has finished reading it.
//
// With row statistics (`sumsq_mc`), each rank's slice is whole rows: one warp
// reduces a row, sums the squares of the (rounded) sums in fp32 and stores
// that row's sum of squares to every rank with one multimem.st -- the
// statistic the next RMSNorm needs, so no separate row-statistics pass reads
// the reduced rows again.
//
// The epoch is a per-block counter kept in the signal pad (so a captured CUDA
// graph replays correctly): block b of call k on every rank uses epoch k of
// block b.  Waits compare with wrap-safe arithmetic and give up after
// kWaitLimitNs, OR-ing TH_DEVERR_MBAR_TIMEOUT into the device error word and
// skipping the rest of the block's work.
//
// The reference runs its collectives through NCCL from Python; this kernel
// replaces the all-reduce after the row-split projections of the
// tensor-parallel Llama block (o_proj and down_proj).
#include "common.cuh"

namespace th {

constexpr int kArMaxCtas = TH_ALLREDUCE_MAX_CTAS;
constexpr int kArMaxWorld = TH_ALLREDUCE_MAX_WORLD;
constexpr int kArThreads = 512;
constexpr int kArWarps = kArThreads / 32;
constexpr int kArUnroll = 4;

// Signal pad layout (uint32 words): [2 phases][kArMaxCtas blocks][kArMaxWorld sources], then the
// per-block epoch counters [kArMaxCtas].
static_assert(TH_ALLREDUCE_SIGNAL_BYTES >= (2 * kArMaxCtas * kArMaxWorld + kArMaxCtas) * 4, "signal pad too small");

struct ArParams {
  uint8_t* mc;                   // multicast address of the range's first byte
  uint32_t* const* peer_sig;     // [world] every rank's signal pad, as mapped here
  uint32_t* sig;                 // this rank's signal pad
  int64_t slice_vecs;            // 16-byte vectors per rank slice
  int32_t rank, world, dtype;
  float* sumsq_mc;               // row statistics: multicast address of the fp32 [rows] array (or null)
  int64_t row_vecs;              // 16-byte vectors per row (row statistics)
  int64_t row0;                  // index of this rank's first row in the sumsq array
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

// Thread t (< world) of block b: signal rank t, then wait for rank t's signal.
__device__ bool ar_handshake(const ArParams& p, int phase, int t, uint32_t epoch) {
  const int64_t slot = ((int64_t)phase * kArMaxCtas + blockIdx.x) * kArMaxWorld;
  fence_proxy_alias();
  st_release_sys(p.peer_sig[t] + slot + p.rank, epoch);
  const uint32_t* mine = p.sig + slot + t;
  if ((int32_t)(ld_acquire_sys(mine) - epoch) >= 0) return true;
  const unsigned long long t0 = globaltimer_ns();
  while ((int32_t)(ld_acquire_sys(mine) - epoch) < 0) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      atomicOr(&g_device_error, TH_DEVERR_MBAR_TIMEOUT);
      return false;
    }
  }
  fence_proxy_alias();
  return true;
}

template <int DTYPE>
__device__ __forceinline__ uint4 mm_ld_reduce(const uint8_t* a) {
  uint4 v;
  if constexpr (DTYPE == TH_BF16) {
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(a)
                 : "memory");
  } else if constexpr (DTYPE == TH_F16) {
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(a)
                 : "memory");
  } else {
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(a)
                 : "memory");
  }
  return v;
}

template <int DTYPE>
__device__ __forceinline__ void mm_st(uint8_t* a, uint4 v) {
  if constexpr (DTYPE == TH_BF16) {
    asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1,%2,%3,%4};" ::"l"(a), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
  } else if constexpr (DTYPE == TH_F16) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f16x2 [%0], {%1,%2,%3,%4};" ::"l"(a), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
  } else {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(a), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
  }
}

__device__ __forceinline__ void mm_st_f32(float* a, float v) {
  asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(a), "f"(v) : "memory");
}

// Sum of squares of the 16-byte vector's elements (fp32).
template <int DTYPE>
__device__ __forceinline__ float sumsq16(uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (DTYPE == TH_BF16) {
      const float lo = __uint_as_float(w[i] << 16), hi = __uint_as_float(w[i] & 0xffff0000u);
      s = fmaf(lo, lo, fmaf(hi, hi, s));
    } else if constexpr (DTYPE == TH_F16) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      s = fmaf(f.x, f.x, fmaf(f.y, f.y, s));
    } else {
      const float f = __uint_as_float(w[i]);
      s = fmaf(f, f, s);
    }
  }
  return s;
}

// This rank's slice, one warp per row, with the row's sum of squares stored to every rank.
template <int DTYPE>
__device__ __forceinline__ void reduce_rows(const ArParams& p, uint8_t* base) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rows = p.slice_vecs / p.row_vecs;
  for (int64_t r = (int64_t)blockIdx.x * kArWarps + warp; r < rows; r += (int64_t)gridDim.x * kArWarps) {
    uint8_t* row = base + r * p.row_vecs * 16;
    float ss = 0.f;
    int64_t i = lane;
    for (; i + (kArUnroll - 1) * 32 < p.row_vecs; i += kArUnroll * 32) {
      uint4 v[kArUnroll];
#pragma unroll
      for (int u = 0; u < kArUnroll; ++u) v[u] = mm_ld_reduce<DTYPE>(row + (i + u * 32) * 16);
#pragma unroll
      for (int u = 0; u < kArUnroll; ++u) {
        mm_st<DTYPE>(row + (i + u * 32) * 16, v[u]);
        ss += sumsq16<DTYPE>(v[u]);
      }
    }
    for (; i < p.row_vecs; i += 32) {
      const uint4 v = mm_ld_reduce<DTYPE>(row + i * 16);
      mm_st<DTYPE>(row + i * 16, v);
      ss += sumsq16<DTYPE>(v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) mm_st_f32(p.sumsq_mc + p.row0 + r, ss);
  }
}

template <int DTYPE>
__global__ void __launch_bounds__(kArThreads) allreduce_mm_kernel(ArParams p) {
  __shared__ int s_ok;
  __shared__ uint32_t s_epoch;
  const int tid = threadIdx.x;
  uint32_t* counter = p.sig + 2 * kArMaxCtas * kArMaxWorld + blockIdx.x;
  if (tid == 0) {
    s_ok = 1;
    s_epoch = *counter + 1;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  if (tid < p.world && !ar_handshake(p, 0, tid, epoch)) s_ok = 0;
  __syncthreads();
  if (s_ok && p.sumsq_mc) {
    reduce_rows<DTYPE>(p, p.mc + (int64_t)p.rank * p.slice_vecs * 16);
  } else if (s_ok) {
    // rank r's slice, vectors spread over the grid; kArUnroll loads in flight per thread
    uint8_t* base = p.mc + (int64_t)p.rank * p.slice_vecs * 16;
    const int64_t stride = (int64_t)gridDim.x * kArThreads;
    int64_t i = (int64_t)blockIdx.x * kArThreads + tid;
    for (; i + (kArUnroll - 1) * stride < p.slice_vecs; i += kArUnroll * stride) {
      uint4 v[kArUnroll];
#pragma unroll
      for (int u = 0; u < kArUnroll; ++u) v[u] = mm_ld_reduce<DTYPE>(base + (i + u * stride) * 16);
#pragma unroll
      for (int u = 0; u < kArUnroll; ++u) mm_st<DTYPE>(base + (i + u * stride) * 16, v[u]);
    }
    for (; i < p.slice_vecs; i += stride) mm_st<DTYPE>(base + i * 16, mm_ld_reduce<DTYPE>(base + i * 16));
  }
  __syncthreads();
  if (!s_ok) return;  // block-uniform: the start handshake gave up
  if (tid < p.world && !ar_handshake(p, 1, tid, epoch)) s_ok = 0;
  __syncthreads();
  if (tid == 0) *counter = epoch;  // the next call of this block uses epoch + 1
}

}  // namespace th

extern "C" int th_allreduce(const th_allreduce_args* a, void* stream) {
  using namespace th;
  if (!a) return fail(TH_EINVAL, "th_allreduce: args is NULL");
  if (!a->mc || !a->peer_sig || !a->sig) return fail(TH_EINVAL, "th_allreduce: mc, peer_sig and sig are required");
  if (a->world < 1 || a->world > kArMaxWorld || a->rank < 0 || a->rank >= a->world)
    return fail(TH_EINVAL, "th_allreduce: rank %d / world %d (world must be in [1, %d])", a->rank, a->world, kArMaxWorld);
  const int ctas = a->ctas > 0 ? a->ctas : 32;
  if (ctas > kArMaxCtas) return fail(TH_EINVAL, "th_allreduce: ctas %d > %d", ctas, kArMaxCtas);
  const int64_t esz = a->dtype == TH_F32 ? 4 : (a->dtype == TH_BF16 || a->dtype == TH_F16) ? 2 : 0;
  if (!esz) return fail(TH_EDTYPE, "th_allreduce: dtype %d (bf16, f16 or f32)", a->dtype);
  if (a->offset < 0 || a->bytes < 0) return fail(TH_EINVAL, "th_allreduce: negative offset or size");
  if (a->bytes % (16 * (int64_t)a->world) != 0)
    return fail(TH_EALIGN, "th_allreduce: %lld bytes is not a multiple of 16 x world", (long long)a->bytes);
  uint8_t* mc = static_cast<uint8_t*>(a->mc) + a->offset;
  if (!aligned16(mc) || !aligned16(a->sig)) return fail(TH_EALIGN, "th_allreduce: range or signal pad not 16-byte aligned");
  if (a->sumsq_mc) {  // row statistics: every rank's slice is whole rows
    if (a->row_bytes <= 0 || a->row_bytes % 16 != 0 || a->offset % a->row_bytes != 0 ||
        a->bytes % (a->row_bytes * a->world) != 0)
      return fail(TH_EINVAL, "th_allreduce: row statistics need whole rows per rank (row_bytes %lld, offset %lld, "
                  "bytes %lld, world %d)", (long long)a->row_bytes, (long long)a->offset, (long long)a->bytes, a->world);
    if (reinterpret_cast<uintptr_t>(a->sumsq_mc) % 4 != 0) return fail(TH_EALIGN, "th_allreduce: sumsq_mc misaligned");
  }
  if (a->bytes == 0 || a->world == 1) return TH_OK;
  ArParams p;
  p.mc = mc;
  p.peer_sig = reinterpret_cast<uint32_t* const*>(a->peer_sig);
  p.sig = static_cast<uint32_t*>(a->sig);
  p.slice_vecs = a->bytes / 16 / a->world;
  p.rank = a->rank;
  p.world = a->world;
  p.dtype = a->dtype;
  p.sumsq_mc = a->sumsq_mc;
  p.row_vecs = a->sumsq_mc ? a->row_bytes / 16 : 0;
  p.row0 = a->sumsq_mc ? a->offset / a->row_bytes + (int64_t)a->rank * (a->bytes / a->world / a->row_bytes) : 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (a->dtype) {
    case TH_BF16: allreduce_mm_kernel<TH_BF16><<<ctas, kArThreads, 0, st>>>(p); break;
    case TH_F16: allreduce_mm_kernel<TH_F16><<<ctas, kArThreads, 0, st>>>(p); break;
    default: allreduce_mm_kernel<TH_F32><<<ctas, kArThreads, 0, st>>>(p); break;
  }
  return check_launch("th_allreduce");
}
