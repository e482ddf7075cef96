// th_gemm: one reference `gemm` KernelSpec (shared LHS, sibling GEMMs
// concatenated along N, RMSNorm row-scale fold, fused epilogue) on B200.
//
//   bf16 / fp16: tcgen05.mma (kind::f16, M=128, N=BN) with the accumulator
//                in TMEM.  A 4-6 stage shared-memory ring is filled by TMA
//                (128-byte swizzle, no multicast); one thread issues TMA,
//                one thread issues MMAs, tcgen05.commit frees ring slots.
//   fp32:        FFMA tiles (fp32 models need fp32 accuracy, which the
//                tensor cores' tf32 mode does not give).
// Both stage the accumulator tile in shared memory and run the same
// epilogue (row scale, activation segment, RoPE, SwiGLU, residual, stores,
// sum-of-squares partials), so the two paths have identical semantics.
#include <cstdlib>
#include <cstring>

#include "common.cuh"

namespace th {

struct EpiParams {
  void* d;
  int64_t ldd;
  int m, n;  // n = accumulator columns (W rows)
  const float* rs_parts;
  int rs_nparts;
  float rs_inv_k, rs_eps;
  int act, act_begin, act_end;
  const float* bias;
  const float* rope_cos;
  const float* rope_sin;
  int rope_begin, rope_end, rope_hd, rope_seq;
  int rope_vec;  // tables 16-byte aligned and head_dim % 4 == 0: 16-byte table loads
  int rs_vec;    // row-scale parts 16-byte aligned with a multiple of 4 per row: 16-byte loads
  int swiglu;
  const void* residual;
  int64_t ld_res;
  float* out2;
  int64_t ld_out2;
  int tail_begin;  // in output columns; >= n_out means none
  float* ss_out;
  int64_t ss_ld;
  int tma_store;  // tcgen05 kernels: 32 x 32 output chunks leave through shared memory and a TMA store
  int d_cols;     // columns of d the TMA store map covers (min(n_out, tail_begin))
  int res_tma;    // residual kernels: the residual chunk arrives by TMA into the same staging buffer
};

// The activation of an activation segment (TH_ACT_*): torch's silu, softplus
// (threshold 20) and gelu in its erf and tanh forms.
__device__ __forceinline__ float act_apply(int act, float x) {
  switch (act) {
    case TH_ACT_SILU: return silu_f(x);
    case TH_ACT_SOFTPLUS: return softplus_f(x);
    case TH_ACT_GELU: return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
    case TH_ACT_GELU_TANH: {
      const float u = 0.79788456080286536f * (x + 0.044715f * x * x * x);  // sqrt(2/pi) (x + 0.044715 x^3)
      return 0.5f * x * (1.0f + tanhf(u));
    }
    default: return x;
  }
}

// Accumulator value at (local row rl, local col j) with the row scale.
__device__ __forceinline__ float acc_at(const float* tile, int ldt, int rl, int j, float rs) {
  return tile[rl * ldt + j] * rs;
}

// Run the epilogue of one BM x BN accumulator tile that sits in shared
// memory (fp32, row stride ldt).  All NT threads of the CTA participate.
// rscale[BM] is scratch for the per-row scale.
template <typename T, int NT, int BM, int BN>
__device__ void epilogue_tile(const float* tile, int ldt, float* rscale, const EpiParams& ep, int m0, int n0) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NW = NT / 32;
  // 1. per-row scale
  for (int rl = tid; rl < BM; rl += NT) {
    float r = 1.0f;
    int row = m0 + rl;
    if (ep.rs_parts && row < ep.m) {
      const float* p = ep.rs_parts + (int64_t)row * ep.rs_nparts;
      float s = 0.f;
      for (int i = 0; i < ep.rs_nparts; ++i) s += p[i];
      r = rsqrtf(s * ep.rs_inv_k + ep.rs_eps);
    }
    rscale[rl] = r;
  }
  __syncthreads();
  const int bn_out = ep.swiglu ? BN / 2 : BN;
  const int n_out = ep.swiglu ? ep.n / 2 : ep.n;
  const int o0 = ep.swiglu ? n0 / 2 : n0;  // first output column of the tile
  T* d = reinterpret_cast<T*>(ep.d);
  const T* res = reinterpret_cast<const T*>(ep.residual);
  for (int rl = warp; rl < BM; rl += NW) {
    const int row = m0 + rl;
    if (row >= ep.m) break;
    const float rs = rscale[rl];
    for (int base = 0; base < bn_out; base += 256) {  // warp-uniform trip count (shuffles below)
      const int ol = base + lane * 8;
      const int oc = o0 + ol;  // global output column of v[0]
      float v[8];
      const bool live = ol < bn_out && oc < n_out;
      if (live) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int jo = ol + e;
          float x;
          if (ep.swiglu) {
            const int g = jo >> 6, w = jo & 63;
            x = silu_f(acc_at(tile, ldt, rl, g * 128 + w, rs)) * acc_at(tile, ldt, rl, g * 128 + 64 + w, rs);
          } else {
            const int c = oc + e;
            x = acc_at(tile, ldt, rl, jo, rs);
            if ((ep.act != TH_ACT_NONE || ep.bias) && c >= ep.act_begin && c < ep.act_end) {
              if (ep.bias) x += ep.bias[c - ep.act_begin];
              x = act_apply(ep.act, x);
            }
            if (ep.rope_cos && c >= ep.rope_begin && c < ep.rope_end) {
              const int hd = ep.rope_hd, half = hd >> 1;
              const int within = (c - ep.rope_begin) % hd;
              const int partner = within < half ? jo + half : jo - half;
              const float pv = acc_at(tile, ldt, rl, partner, rs);
              const float rot = within < half ? -pv : pv;
              const int64_t t = (int64_t)(row % ep.rope_seq) * hd + within;
              x = x * ep.rope_cos[t] + rot * ep.rope_sin[t];
            }
          }
          v[e] = x;
        }
      }
      float ss = 0.f;
      if (live) {
        if (oc >= ep.tail_begin) {
          // fp32 tail (tail_begin is a multiple of 8, so a vector never straddles it)
          float* o2 = ep.out2 + (int64_t)row * ep.ld_out2 + (oc - ep.tail_begin);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (oc + e < n_out) o2[e] = v[e];
        } else {
          if (res) {
            float r8[8];
            load8<T>(res + (int64_t)row * ep.ld_res + oc, r8);
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] += r8[e];
          }
          ss = store8_ss<T>(d + (int64_t)row * ep.ldd + oc, v);
        }
      }
      if (ep.ss_out) {
        // 8 lanes x 8 columns = one 64-column group
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        ss += __shfl_xor_sync(0xffffffffu, ss, 4);
        if ((lane & 7) == 0 && live && oc < ep.tail_begin) ep.ss_out[(int64_t)row * ep.ss_ld + (oc >> 6)] = ss;
      }
    }
  }
}

// ------------------------------------------------------------ tcgen05 path
// Persistent, warp-specialised kernel (320 threads, one CTA per SM):
//   warp 0  TMA producer: A/B tiles (128-byte swizzle) into a STAGES-deep ring
//   warp 1  MMA issuer:   tcgen05.mma 128xBNx16 into one of two TMEM accumulators
//   warps 2-9 epilogue:   thread = accumulator row, two warps per TMEM lane
//           quarter splitting the tile's columns; tcgen05.ld 32 columns at a
//           time, all fused stages in registers, direct stores
// The two accumulators (2*BN TMEM columns) let the epilogue of tile i overlap
// the mainloop of tile i+1.  Every wait is bounded (mbar_wait): a stuck
// pipeline sets the device error word and the kernel drains and exits.
// Tile order of the persistent kernels: groups of 8 row tiles walked column
// by column, so the tiles in flight (one per CTA or CTA pair) share a few row
// tiles of A and one band of B rows, both L2-resident even when B alone is
// larger than L2 (a 28672 x 4096 gate|up weight is 235 MB).
__device__ __forceinline__ int2 tile_coords(int tile, int tiles_m, int tiles_n) {
  constexpr int GM = 8;
  const int per_group = GM * tiles_n;
  const int g = tile / per_group, r = tile - g * per_group;
  const int rows_left = tiles_m - g * GM;
  const int gm = rows_left < GM ? rows_left : GM;
  return make_int2(g * GM + r % gm, r / gm);  // (row tile, column tile)
}

// Output staging of the tcgen05 epilogue: every epilogue warp owns two 2 KB
// buffers (32 rows x 64 bytes) in shared memory after the operand ring.
constexpr int EPI_WARPS = 8, EPI_BUF_BYTES = 2048;
constexpr int EPI_STAGE_BYTES = EPI_WARPS * 2 * EPI_BUF_BYTES;

template <int BN>
struct TcCfg {
  static constexpr int BM = 128, BK = 64;
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  // ring | barriers (1 KB) | output staging (EPI_STAGE_BYTES)
  static constexpr int STAGE_OFF = RING_BYTES + 1024;
  static constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGE_OFF + EPI_STAGE_BYTES;
};

// Residual add, store, fp32 tail and sum-of-squares partials of a 32-value
// row chunk whose first element is output column `oc`.  Returns the chunk's
// sum of squares of the stored (rounded) values (0 when the GEMM has no
// sum-of-squares output).
template <typename T>
__device__ __forceinline__ float finish_chunk(float* v, int row, int oc, int n_out, const EpiParams& ep) {
  T* d = reinterpret_cast<T*>(ep.d);
  const T* res = reinterpret_cast<const T*>(ep.residual);
  const bool want_ss = ep.ss_out != nullptr;
  float ss = 0.f;
#pragma unroll
  for (int e8 = 0; e8 < 32; e8 += 8) {
    const int c = oc + e8;
    if (c >= n_out) break;
    if (c >= ep.tail_begin) {
      float* o2 = ep.out2 + (int64_t)row * ep.ld_out2 + (c - ep.tail_begin);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (c + e < n_out) o2[e] = v[e8 + e];
      continue;
    }
    if (res) {
      float r8[8];
      load8<T>(res + (int64_t)row * ep.ld_res + c, r8);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e8 + e] += r8[e];
    }
    if (want_ss) ss += store8_ss<T>(d + (int64_t)row * ep.ldd + c, v + e8);
    else store8<T>(d + (int64_t)row * ep.ldd + c, v + e8);
  }
  return ss;
}

struct OutStage {
  uint8_t* buf;             // this warp's two buffers
  const CUtensorMap* map;   // d as [rows, d_cols], box 32 x 32, 64-byte swizzle
  uint32_t n;               // stores this warp has issued
  const CUtensorMap* rmap;  // the residual, same geometry (res_tma)
  uint64_t* bar;            // one mbarrier per buffer: the residual chunk loaded into it has landed
  uint32_t loads;           // residual loads lane 0 has issued (chunk n's is the n-th)
};

// 8 values rounded to T and packed into 16 bytes; returns their sum of squares (of the rounded values).
template <typename T>
__device__ __forceinline__ float pack8_ss(const float* v, uint4& u) {
  float s = 0.f;
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f;
    if constexpr (DT<T>::id == TH_BF16) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
      f = __bfloat1622float2(h);
    } else {
      __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
      f = __half22float2(h);
    }
    s = fmaf(f.x, f.x, fmaf(f.y, f.y, s));
  }
  return s;
}

// A warp's 32 rows x 32 columns of output (lane = row row0 + lane, its 32
// values from column oc) leave through shared memory and one TMA store:
// every lane writes its row as four 16-byte pieces in the layout of the
// map's 64-byte swizzle (piece j of row r at slot j ^ ((r >> 1) & 3), so the
// 32 rows of one store instruction fall on distinct bank groups eight rows at
// a time), then lane 0 issues the store.  The buffer written here was last
// read by the store two calls ago; rows and columns outside d are clipped by
// the TMA unit.  All 32 lanes must call it.  Returns the lane's sum of
// squares of the stored values.
template <typename T>
__device__ __forceinline__ float stage_store32(const float* v, OutStage& st, int oc, int row0, int lane) {
  uint8_t* buf = st.buf + (st.n & 1) * EPI_BUF_BYTES;
  if (lane == 0) bulk_wait_read1();
  __syncwarp();
  const uint32_t row_addr = smem_u32(buf) + (uint32_t)lane * 64u;
  const int sw = (lane >> 1) & 3;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 u;
    ss += pack8_ss<T>(v + 8 * j, u);
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(row_addr + 16u * (uint32_t)(j ^ sw)), "r"(u.x),
                 "r"(u.y), "r"(u.z), "r"(u.w)
                 : "memory");
  }
  fence_proxy_async();  // the generic-proxy writes above, before the async-proxy read of the store
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(st.map, buf, oc, row0);
    bulk_commit();
  }
  ++st.n;
  return ss;
}

// Lane 0: TMA-load the residual chunk (rows row0.., columns oc..) into buffer b of this warp.
__device__ __forceinline__ void res_load32(OutStage& st, int b, int oc, int row0) {
  mbar_arrive_expect_tx(&st.bar[b], EPI_BUF_BYTES);
  tma_load_2d(st.buf + b * EPI_BUF_BYTES, st.rmap, &st.bar[b], oc, row0);
  ++st.loads;
}

// Lane 0, as the warp leaves the epilogue: residual loads it issued that no chunk consumed (after a
// wait gave up) land before the CTA ends; the wait is bounded as well.
__device__ __forceinline__ void res_drain(OutStage& st) {
  volatile int quit = 0;
  for (uint32_t k = st.n; k < st.loads; ++k)
    if (!mbar_wait_for(&st.bar[k & 1], (k >> 1) & 1, &quit, 100000000ull)) break;
}

// stage_store32 for a chunk whose residual sits in the buffer (res_load32): each lane adds its row
// of the residual and writes the sums back in place, then lane 0 stores the buffer.  `want_ss`: sum
// of squares of the stored values.  Returns false when the wait for the residual gave up.
template <typename T>
__device__ __forceinline__ bool stage_store32_res(float* v, OutStage& st, int oc, int row0, int lane, float& ss,
                                                  volatile int* abort_flag) {
  const int b = st.n & 1;
  uint8_t* buf = st.buf + b * EPI_BUF_BYTES;
  if (!mbar_wait(&st.bar[b], (st.n >> 1) & 1, abort_flag)) return false;
  const uint32_t row_addr = smem_u32(buf) + (uint32_t)lane * 64u;
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t a = row_addr + 16u * (uint32_t)(j ^ sw);
    uint4 u;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w) : "r"(a));
    const T* rh = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[8 * j + e] += to_f32(rh[e]);
    ss += pack8_ss<T>(v + 8 * j, u);
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(u.x), "r"(u.y), "r"(u.z), "r"(u.w)
                 : "memory");
  }
  fence_proxy_async();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(st.map, buf, oc, row0);
    bulk_commit();
  }
  ++st.n;
  return true;
}

// Whether the 32-column chunk at output column oc goes out through stage_store32 (warp-uniform).
__device__ __forceinline__ bool staged(const EpiParams& ep, int oc) {
  return ep.tma_store && oc < ep.d_cols && oc + 32 <= ep.tail_begin;
}

// Residual of a 32-column chunk added to v (16-byte loads of this lane's row).
template <typename T>
__device__ __forceinline__ void add_residual32(float* v, int row, int oc, const EpiParams& ep) {
  const T* res = reinterpret_cast<const T*>(ep.residual) + (int64_t)row * ep.ld_res + oc;
#pragma unroll
  for (int e8 = 0; e8 < 4; ++e8) {
    if (oc + e8 * 8 >= ep.d_cols) break;  // n_out % 8 == 0: a piece is wholly inside or outside
    float r8[8];
    load8<T>(res + e8 * 8, r8);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e8 * 8 + e] += r8[e];
  }
}

// Epilogue variants compiled as separate kernels (smaller code per kernel).
constexpr int EPI_ROPE = 1, EPI_SWIGLU = 2, EPI_RES = 4;

// Residual of one 32-column chunk of this thread's row, as raw 16-byte loads.
template <typename T>
__device__ __forceinline__ void res_issue(uint4 (&r)[4], int row, bool row_ok, int col, const EpiParams& ep) {
  const T* res = reinterpret_cast<const T*>(ep.residual) + (int64_t)row * ep.ld_res;
#pragma unroll
  for (int e8 = 0; e8 < 4; ++e8) {
    const int c = col + e8 * 8;
    r[e8] = (row_ok && c < ep.tail_begin && c < ep.n) ? *reinterpret_cast<const uint4*>(res + c) : make_uint4(0, 0, 0, 0);
  }
}

// Residual epilogue (plain GEMM + residual, optional row scale / activation):
// the residual of chunk c+2 is in flight while chunk c is stored, and the
// first two chunks were issued before the accumulator was ready.
template <typename T, int NC>
__device__ __forceinline__ bool epilogue_row_res(uint32_t tbase, int row, bool row_ok, float rs, int n0, int cb,
                                                 const EpiParams& ep, uint4 (&rb)[3][4], OutStage& ost, int row0,
                                                 int lane, volatile int* abort_flag) {
  const int n_out = ep.n;
  T* d = reinterpret_cast<T*>(ep.d);
  const bool want_ss = ep.ss_out != nullptr;
  float ss = 0.f;
  if (ep.res_tma) {
    // the residual of chunks 0 and 1 was loaded into this warp's two buffers before the accumulator
    // was ready; chunk ci + 2 is loaded into chunk ci's buffer once chunk ci's store has read it
    for (int ci = 0; ci < NC; ++ci) {
      const int c = cb + ci * 32, col = n0 + c;
      if (col < ep.d_cols) {  // else past the output (last column tile); the sum-of-squares group still closes
        float v[32];
        tmem_ld32(tbase + c, v);
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] *= rs;
        if ((ep.act != TH_ACT_NONE || ep.bias) && col < ep.act_end && col + 32 > ep.act_begin) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int cc = col + e;
            if (cc >= ep.act_begin && cc < ep.act_end) {
              float x = v[e] + (ep.bias ? ep.bias[cc - ep.act_begin] : 0.f);
              v[e] = act_apply(ep.act, x);
            }
          }
        }
        const int b = ost.n & 1;
        float s32 = 0.f;
        if (!stage_store32_res<T>(v, ost, col, row0, lane, s32, abort_flag)) return false;
        if (want_ss) ss += s32;
        if (lane == 0 && ci + 2 < NC && col + 64 < ep.d_cols) {
          bulk_wait_read0();  // the store just issued has read the buffer
          res_load32(ost, b, col + 64, row0);
        }
        __syncwarp();
      }
      if ((ci & 1) == 1) {
        const int g0 = col - 32;
        if (ep.ss_out && row_ok && g0 < n_out) ep.ss_out[(int64_t)row * ep.ss_ld + (g0 >> 6)] = ss;
        ss = 0.f;
      }
    }
    return true;
  }
#pragma unroll
  for (int ci = 0; ci < NC; ++ci) {
    const int c = cb + ci * 32, col = n0 + c;
    if (ci + 2 < NC) res_issue<T>(rb[(ci + 2) % 3], row, row_ok, col + 64, ep);
    float v[32];
    tmem_ld32(tbase + c, v);
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] *= rs;
    if ((ep.act != TH_ACT_NONE || ep.bias) && col < ep.act_end && col + 32 > ep.act_begin) {
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int cc = col + e;
        if (cc >= ep.act_begin && cc < ep.act_end) {
          float x = v[e] + (ep.bias ? ep.bias[cc - ep.act_begin] : 0.f);
          v[e] = act_apply(ep.act, x);
        }
      }
    }
    if (staged(ep, col)) {  // the whole warp: residual from the prefetched registers, then shared memory + TMA
#pragma unroll
      for (int e8 = 0; e8 < 4; ++e8) {
        const uint4 u = rb[ci % 3][e8];
        const T* rh = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e8 * 8 + e] += to_f32(rh[e]);
      }
      const float s32 = stage_store32<T>(v, ost, col, row0, lane);
      if (want_ss) ss += s32;
    } else if (row_ok) {
#pragma unroll
      for (int e8 = 0; e8 < 4; ++e8) {
        const int cc = col + e8 * 8;
        if (cc >= n_out) break;
        if (cc >= ep.tail_begin) {
          float* o2 = ep.out2 + (int64_t)row * ep.ld_out2 + (cc - ep.tail_begin);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (cc + e < n_out) o2[e] = v[e8 * 8 + e];
          continue;
        }
        const uint4 u = rb[ci % 3][e8];
        const T* rh = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e8 * 8 + e] += to_f32(rh[e]);
        if (want_ss) ss += store8_ss<T>(d + (int64_t)row * ep.ldd + cc, v + e8 * 8);
        else store8<T>(d + (int64_t)row * ep.ldd + cc, v + e8 * 8);
      }
    }
    if ((ci & 1) == 1) {
      const int g0 = col - 32;  // first column of this 64-column group
      if (ep.ss_out && row_ok && g0 < n_out && g0 < ep.tail_begin) ep.ss_out[(int64_t)row * ep.ss_ld + (g0 >> 6)] = ss;
      ss = 0.f;
    }
  }
  return true;
}

// Epilogue of one accumulator row (this thread) of a 128 x BN tile.
template <typename T, int BN, int EPI>
__device__ __forceinline__ void epilogue_row(uint32_t tbase, int row, bool row_ok, float rs, int n0, int cb, int ce,
                                             const EpiParams& ep, OutStage& ost, int row0, int lane) {
  if constexpr ((EPI & EPI_SWIGLU) != 0) {
    const int n_out = ep.n / 2;
    for (int g = cb / 128; g < ce / 128; ++g) {
      float ss = 0.f;
      for (int q = 0; q < 2; ++q) {
        float gv[32], uv[32];
        tmem_ld32(tbase + g * 128 + q * 32, gv);
        tmem_ld32(tbase + g * 128 + 64 + q * 32, uv);
#pragma unroll
        for (int e = 0; e < 32; ++e) gv[e] = silu_f(gv[e] * rs) * (uv[e] * rs);
        const int oc = n0 / 2 + g * 64 + q * 32;
        if (staged(ep, oc)) {
          const float s32 = stage_store32<T>(gv, ost, oc, row0, lane);
          if (ep.ss_out) ss += s32;
        } else if (row_ok) {
          ss += finish_chunk<T>(gv, row, oc, n_out, ep);
        }
      }
      const int oc = n0 / 2 + g * 64;
      if (ep.ss_out && row_ok && oc < n_out) ep.ss_out[(int64_t)row * ep.ss_ld + (oc >> 6)] = ss;
    }
    return;
  }
  const int n_out = ep.n;
  float ss = 0.f;
  for (int c = cb; c < ce; c += 32) {
    float v[32];
    tmem_ld32(tbase + c, v);
    const int col = n0 + c;
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] *= rs;
    if ((ep.act != TH_ACT_NONE || ep.bias) && col < ep.act_end && col + 32 > ep.act_begin) {
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int cc = col + e;
        if (cc >= ep.act_begin && cc < ep.act_end) {
          float x = v[e] + (ep.bias ? ep.bias[cc - ep.act_begin] : 0.f);
          v[e] = act_apply(ep.act, x);
        }
      }
    }
    if constexpr ((EPI & EPI_ROPE) == 0) {
    } else if (col < ep.rope_end && col + 32 > ep.rope_begin) {
      const int hd = ep.rope_hd, half = hd >> 1;
      const int64_t pos = row_ok ? (int64_t)(row % ep.rope_seq) * hd : 0;
      if (half >= 32) {  // the partner 32 columns are a whole chunk away
        const int within0 = (col - ep.rope_begin) % hd;
        const bool first = within0 < half;
        float pv[32];
        tmem_ld32(tbase + (first ? c + half : c - half), pv);
        if (ep.rope_vec) {
          // each lane (row) reads its own table row: 16-byte loads cut the cache lines a warp
          // touches per table element fourfold, which bounded the QKV GEMM's epilogue
          const float4* c4 = reinterpret_cast<const float4*>(ep.rope_cos + pos + within0);
          const float4* s4 = reinterpret_cast<const float4*>(ep.rope_sin + pos + within0);
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4) {
            const float4 cq = __ldg(c4 + q4), sq = __ldg(s4 + q4);
            const float cv[4] = {cq.x, cq.y, cq.z, cq.w}, sv[4] = {sq.x, sq.y, sq.z, sq.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int k = q4 * 4 + e;
              const float rot = first ? -pv[k] * rs : pv[k] * rs;
              v[k] = v[k] * cv[e] + rot * sv[e];
            }
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float rot = first ? -pv[e] * rs : pv[e] * rs;
            v[e] = v[e] * ep.rope_cos[pos + within0 + e] + rot * ep.rope_sin[pos + within0 + e];
          }
        }
      } else {  // heads of <= 32 columns: partner inside this chunk
        float t[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) t[e] = v[e];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int within = (col + e - ep.rope_begin) % hd;
          const bool first = within < half;
          const float pv = first ? t[(e + half) & 31] : t[(e - half) & 31];
          v[e] = t[e] * ep.rope_cos[pos + within] + (first ? -pv : pv) * ep.rope_sin[pos + within];
        }
      }
    }
    if (staged(ep, col)) {
      if (ep.residual && row_ok) add_residual32<T>(v, row, col, ep);
      const float s32 = stage_store32<T>(v, ost, col, row0, lane);
      if (ep.ss_out) ss += s32;
    } else if (row_ok) {
      ss += finish_chunk<T>(v, row, col, n_out, ep);
    }
    if (((c + 32) & 63) == 0) {
      const int g0 = col - 32;  // first column of this 64-column group
      if (ep.ss_out && row_ok && g0 < n_out && g0 < ep.tail_begin) ep.ss_out[(int64_t)row * ep.ss_ld + (g0 >> 6)] = ss;
      ss = 0.f;
    }
  }
}

// One epilogue warp's share (warps 2..9: two per TMEM lane quarter, each one
// half of the columns) of the 128 x BN accumulator tile at TMEM column
// `tacc` whose first output row is m0: the row scale and the first residual
// chunks are fetched while the accumulator fills, then the rows are finished.
// Returns false when the wait for the accumulator gave up.
template <typename T, int BN, int EPI>
__device__ __forceinline__ bool epilogue_tmem_tile(uint32_t tacc, int warp, int lane, int m0, int n0, uint64_t* tfull,
                                              uint32_t parity, volatile int* abort_flag, const EpiParams& ep,
                                              OutStage& ost) {
  const int q = warp & 3;  // TMEM lane quarter this warp may read
  const int hh = (warp - 2) >> 2;
  const int rl = q * 32 + lane;
  // a head of RoPE or a 128-column gate|up block must not straddle the halves
  constexpr bool split = !((EPI & EPI_SWIGLU) != 0 && BN < 256);
  const bool rope_whole = (EPI & EPI_ROPE) != 0 && ep.rope_hd > BN / 2;
  const bool halves = split && !rope_whole;
  const int cb = halves ? hh * (BN / 2) : 0, ce = halves ? cb + BN / 2 : (hh ? 0 : BN);
  const int row = m0 + rl;
  const bool row_ok = row < ep.m;
  float rs = 1.f;
  if (ep.rs_parts && row_ok && ce > cb) {
    const float* pp = ep.rs_parts + (int64_t)row * ep.rs_nparts;
    float sacc = 0.f;
    if (ep.rs_vec) {  // each lane reads its own row: 16-byte loads touch a quarter of the lines
      float s4[4] = {0.f, 0.f, 0.f, 0.f};
      for (int k = 0; k < ep.rs_nparts; k += 4) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(pp + k));
        s4[0] += v.x;
        s4[1] += v.y;
        s4[2] += v.z;
        s4[3] += v.w;
      }
      sacc = (s4[0] + s4[1]) + (s4[2] + s4[3]);
    } else {
      for (int k = 0; k < ep.rs_nparts; ++k) sacc += pp[k];
    }
    rs = rsqrtf(sacc * ep.rs_inv_k + ep.rs_eps);
  }
  uint4 rb[3][4];
  const int row0 = m0 + q * 32;  // the warp's first row (its TMEM lane quarter)
  if constexpr ((EPI & EPI_RES) != 0) {
    if (ep.res_tma) {  // residual chunks 0 and 1 into this warp's two buffers, once earlier stores read them
      if (lane == 0) {
        bulk_wait_read0();
#pragma unroll
        for (int i = 0; i < 2 && i < BN / 64; ++i)
          if (n0 + cb + 32 * i < ep.d_cols) res_load32(ost, (ost.n + i) & 1, n0 + cb + 32 * i, row0);
      }
      __syncwarp();
    } else {
      res_issue<T>(rb[0], row, row_ok, n0 + cb, ep);
      res_issue<T>(rb[1], row, row_ok, n0 + cb + 32, ep);
    }
  }
  if (!mbar_wait(tfull, parity, abort_flag)) return false;
  __syncwarp();
  tc_fence_after();
  const uint32_t tb = tacc + ((uint32_t)(q * 32) << 16);
  if constexpr ((EPI & EPI_RES) != 0) {
    if (!epilogue_row_res<T, BN / 64>(tb, row, row_ok, rs, n0, cb, ep, rb, ost, row0, lane, abort_flag)) return false;
  } else if (ce > cb) {
    epilogue_row<T, BN, EPI>(tb, row, row_ok, rs, n0, cb, ce, ep, ost, row0, lane);
  }
  tc_fence_before();
  __syncwarp();
  return true;
}

template <typename T, int BN, int EPI>
__global__ void __launch_bounds__(320, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmR, EpiParams ep,
                   int K, int tiles_m, int tiles_n) {
  using C = TcCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align<1024>(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::RING_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* ebar = reinterpret_cast<uint64_t*>(smem + C::RING_BYTES + 512);  // residual-load barriers, 2 per epilogue warp

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = tiles_m * tiles_n;
  const int nk = (K + C::BK - 1) / C::BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);  // one arrive per epilogue warp
    }
    mbar_init(done, 1);
    for (int b = 0; b < 2 * EPI_WARPS; ++b) mbar_init(&ebar[b], 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (ep.tma_store) tma_prefetch_desc(&tmD);
    if (ep.res_tma) tma_prefetch_desc(&tmR);
  }
  __syncwarp();
  if (warp == 0) tmem_alloc(tmem_slot, C::TMEM_COLS);  // warp-wide .sync.aligned
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // the previous kernel's outputs (this GEMM's operands) are complete
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
        const int2 tc = tile_coords(tile, tiles_m, tiles_n);
        const int m0 = tc.x * C::BM, n0 = tc.y * BN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          uint8_t* sa = smem + s * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
          tma_load_2d(sa, &tmA, &full[s], kb * C::BK, m0);
          tma_load_2d(sa + C::A_BYTES, &tmB, &full[s], kb * C::BK, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      constexpr int fmt = DT<T>::id == TH_BF16 ? 1 : 0;
      int it = 0, i = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++i) {
        const int acc = i & 1, use = i >> 1;
        // the last column tile multiplies only its live columns (N rounded up to 16)
        const int nlive = ep.n - tile_coords(tile, tiles_m, tiles_n).y * BN;
        const int ntile = nlive >= BN ? BN : ((nlive + 15) & ~15);
        const uint32_t idesc = make_idesc_f16(128, ntile, fmt, 0, 0);
        if (!mbar_wait(&tempty[acc], (use & 1) ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
          const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < C::BK / 16; ++k) {
            const uint64_t ad = make_desc_sw128(sa + k * 32, 16, 1024);
            const uint64_t bd = make_desc_sw128(sb + k * 32, 16, 1024);
            tc_mma_f16(d, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          tc_commit(&empty[s]);
        }
        if (ok) tc_commit(&tfull[acc]);
      }
      tc_commit(done);  // tracks every MMA this thread issued
    }
  } else {  // ---- epilogue warps 2..9: two per TMEM lane quarter, each one half of the tile's columns
    OutStage ost{smem + C::STAGE_OFF + (warp - 2) * 2 * EPI_BUF_BYTES, &tmD, 0, &tmR, ebar + 2 * (warp - 2), 0};
    int i = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++i) {
      const int acc = i & 1, use = i >> 1;
      const int2 tc = tile_coords(tile, tiles_m, tiles_n);
      const int m0 = tc.x * C::BM, n0 = tc.y * BN;
      if (!epilogue_tmem_tile<T, BN, EPI>(tmem + (uint32_t)(acc * BN), warp, lane, m0, n0, &tfull[acc], use & 1,
                                          abort_flag, ep, ost))
        break;
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (lane == 0) {
      if (ep.res_tma) res_drain(ost);
      bulk_wait0();  // this warp's output stores are complete before the kernel ends
    }
  }
  __syncwarp();
  // teardown: wait (bounded) for the MMAs to retire before freeing TMEM
  if (threadIdx.x == 64) {
    volatile int dummy = 0;
    mbar_wait(done, 0, &dummy);
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ------------------------------------------------- tcgen05 CTA-pair path
// Cluster of two CTAs on an SM pair computing 256 x BN tiles with
// tcgen05.mma.cta_group::2: each CTA stages its own 128 rows of A and one half
// (BN/2 rows) of B per k-block, so a CTA moves (128 + BN/2) x 64 operands for
// a 128 x BN x 64 product, against (128 + BN) x 64 in the single-CTA kernel.
//   warp 0 (both CTAs)  TMA: its A rows and B half into its own ring; the bytes
//                       are counted on the even CTA's `full` barrier
//   warp 1 (even CTA)   MMA issuer; each ring-slot / accumulator commit arrives
//                       on the barrier of both CTAs
//   warps 2-9 (both)    epilogue of the CTA's 128 rows (its TMEM lanes); the
//                       odd CTA's warps release the accumulator on the even
//                       CTA's `tempty` barrier
// No TMA load multicasts: each CTA loads only its own operands.
template <int BN>
struct Tc2Cfg {
  static constexpr int BM = 128, BK = 64;  // per CTA; the pair's tile is 256 x BN
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = (BN / 2) * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // the ring takes what 227 KB leave after the alignment slack, the barriers and the output staging
  static constexpr int RING_MAX = 227 * 1024 - 2048 - EPI_STAGE_BYTES;
  static constexpr int STAGES = RING_MAX / STAGE_BYTES > 8 ? 8 : RING_MAX / STAGE_BYTES;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * BN <= 256 ? 256 : 512;  // a power of two
  static constexpr int STAGE_OFF = RING_BYTES + 1024;
  static constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGE_OFF + EPI_STAGE_BYTES;
};

template <typename T, int BN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(320, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmR, EpiParams ep,
                    int K, int tiles_m, int tiles_n) {
  using C = Tc2Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align<1024>(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::RING_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* ebar = reinterpret_cast<uint64_t*>(smem + C::RING_BYTES + 512);  // residual-load barriers, 2 per epilogue warp

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int ntiles = tiles_m * tiles_n;
  const int nk = (K + C::BK - 1) / C::BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 16);  // one arrive per epilogue warp of both CTAs
    }
    mbar_init(done, 1);
    for (int b = 0; b < 2 * EPI_WARPS; ++b) mbar_init(&ebar[b], 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (ep.tma_store) tma_prefetch_desc(&tmD);
    if (ep.res_tma) tma_prefetch_desc(&tmR);
  }
  __syncwarp();
  if (warp == 0) tmem_alloc_pair(tmem_slot, C::TMEM_COLS);  // the same warp in both CTAs
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // the previous kernel's outputs (this GEMM's operands) are complete
  pdl_trigger();

  // columns the pair multiplies on a tile (the last column tile: its live
  // columns rounded up to 16); CTA r holds B rows [r * nt / 2, (r + 1) * nt / 2)
  auto tile_cols = [&](int tile) {
    const int nlive = ep.n - tile_coords(tile, tiles_m, tiles_n).y * BN;
    return nlive >= BN ? BN : ((nlive + 15) & ~15);
  };

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer (both CTAs)
      const uint32_t full0 = cluster_addr(full, 0);
      int it = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < ntiles; tile += npairs) {
        const int2 tc = tile_coords(tile, tiles_m, tiles_n);
        const int m0 = tc.x * 2 * C::BM + (int)rank * C::BM;
        const int nb = tc.y * BN + (int)rank * (tile_cols(tile) / 2);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          uint8_t* sa = smem + s * C::STAGE_BYTES;
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * C::STAGE_BYTES);
          const uint32_t fb = full0 + (uint32_t)(s * 8);
          tma_load_2d_pair(sa, &tmA, fb, kb * C::BK, m0);
          tma_load_2d_pair(sa + C::A_BYTES, &tmB, fb, kb * C::BK, nb);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {  // ---- MMA issuer (even CTA)
      constexpr int fmt = DT<T>::id == TH_BF16 ? 1 : 0;
      int it = 0, i = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < ntiles; tile += npairs, ++i) {
        const int acc = i & 1, use = i >> 1;
        const uint32_t idesc = make_idesc_f16(256, tile_cols(tile), fmt, 0, 0);
        if (!mbar_wait(&tempty[acc], (use & 1) ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
          const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < C::BK / 16; ++k) {
            const uint64_t ad = make_desc_sw128(sa + k * 32, 16, 1024);
            const uint64_t bd = make_desc_sw128(sb + k * 32, 16, 1024);
            tc_mma_f16_pair(d, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          tc_commit_pair_both(&empty[s]);
        }
        if (ok) tc_commit_pair_both(&tfull[acc]);
      }
      tc_commit_pair(done);  // tracks every MMA this thread issued
    }
  } else {  // ---- epilogue warps 2..9 (both CTAs): this CTA's 128 rows of the pair's tile
    const uint32_t tempty0 = cluster_addr(tempty, 0);
    OutStage ost{smem + C::STAGE_OFF + (warp - 2) * 2 * EPI_BUF_BYTES, &tmD, 0, &tmR, ebar + 2 * (warp - 2), 0};
    int i = 0;
    for (int tile = pair; tile < ntiles; tile += npairs, ++i) {
      const int acc = i & 1, use = i >> 1;
      const int2 tc = tile_coords(tile, tiles_m, tiles_n);
      const int m0 = tc.x * 2 * C::BM + (int)rank * C::BM, n0 = tc.y * BN;
      if (!epilogue_tmem_tile<T, BN, EPI>(tmem + (uint32_t)(acc * BN), warp, lane, m0, n0, &tfull[acc], use & 1,
                                          abort_flag, ep, ost))
        break;
      if (lane == 0) mbar_arrive_cluster(tempty0 + (uint32_t)(acc * 8));
    }
    if (lane == 0) {
      if (ep.res_tma) res_drain(ost);
      bulk_wait0();  // this warp's output stores are complete before the kernel ends
    }
  }
  __syncwarp();
  // teardown: the even CTA waits (bounded) for its MMAs to retire; then neither
  // CTA frees TMEM or exits while the other may still touch its barriers
  if (leader && threadIdx.x == 64) {
    volatile int dummy = 0;
    mbar_wait(done, 0, &dummy);
  }
  __syncwarp();  // the cluster barrier is .aligned: warps arrive converged
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  if (warp == 0) tmem_dealloc_pair(tmem, C::TMEM_COLS);
}

// --------------------------------------------------------------- FFMA path
constexpr int SM_BM = 32, SM_BN = 128, SM_BK = 16, SM_LDT = SM_BN + 4;

template <typename T>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const T* __restrict__ A, int64_t lda, const T* __restrict__ W,
                                                        int64_t ldw, EpiParams ep, int K) {
  __shared__ float As[SM_BK][SM_BM + 4];
  __shared__ float Ws[SM_BK][SM_BN + 4];
  __shared__ float tile[SM_BM * SM_LDT];
  __shared__ float rscale[SM_BM];
  const int tid = threadIdx.x, tx = tid & 31, ty = tid >> 5;
  const int m0 = blockIdx.y * SM_BM, n0 = blockIdx.x * SM_BN;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += SM_BK) {
    for (int i = tid; i < SM_BM * SM_BK; i += 256) {
      const int r = i / SM_BK, k = i % SM_BK;
      const int gr = m0 + r, gk = k0 + k;
      As[k][r] = (gr < ep.m && gk < K) ? to_f32(A[(int64_t)gr * lda + gk]) : 0.f;
    }
    for (int i = tid; i < SM_BN * SM_BK; i += 256) {
      const int r = i / SM_BK, k = i % SM_BK;
      const int gr = n0 + r, gk = k0 + k;
      Ws[k][r] = (gr < ep.n && gk < K) ? to_f32(W[(int64_t)gr * ldw + gk]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < SM_BK; ++k) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[k][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Ws[k][tx + 32 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) tile[(ty * 4 + i) * SM_LDT + tx + 32 * j] = acc[i][j];
  __syncthreads();
  epilogue_tile<T, 256, SM_BM, SM_BN>(tile, SM_LDT, rscale, ep, m0, n0);
}

// ------------------------------------------------------------------- host
// SMs this launch's persistent grid may occupy: all of them, or the caller's
// sm_limit (at least one CTA pair).
static int gemm_sms(const th_gemm_args* a) {
  const int all = sm_count();
  return a->sm_limit > 0 && a->sm_limit < all ? (a->sm_limit < 2 ? 2 : a->sm_limit) : all;
}

// TH_GEMM_TMA_STORE=0: the tcgen05 epilogue stores each lane's row directly instead of staging
// 32 x 32 chunks in shared memory for a TMA store (for comparisons; read once per process).
static bool tma_store_enabled() {
  static const bool on = [] {
    const char* e = getenv("TH_GEMM_TMA_STORE");
    return !(e && e[0] == '0');
  }();
  return on;
}

// TH_GEMM_TMA_RES=0: residual kernels load the residual with per-lane 16-byte loads instead of TMA.
static bool tma_res_enabled() {
  static const bool on = [] {
    const char* e = getenv("TH_GEMM_TMA_RES");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Copy of the epilogue parameters with the staged output store set up: d as a [m, d_cols] tensor map
// (box 32 x 32, 64-byte swizzle, matching stage_store32), where d_cols = min(n_out, tail_begin); and,
// when every output chunk is staged (d_cols % 32 == 0, no fp32 tail), the residual as a map of the same
// geometry for stage_store32_res.
static int with_out_map(const th_gemm_args* a, const EpiParams& ep, EpiParams* out, CUtensorMap* tm,
                        CUtensorMap* tr) {
  *out = ep;
  const int n_out = a->swiglu ? (int)(a->n / 2) : (int)a->n;
  out->d_cols = ep.tail_begin < n_out ? ep.tail_begin : n_out;
  out->tma_store = 0;
  out->res_tma = 0;
  memset(tm, 0, sizeof(*tm));
  memset(tr, 0, sizeof(*tr));
  if (!tma_store_enabled() || !a->d || out->d_cols < 8) return TH_OK;
  int rc = make_tmap_2d_sw(tm, a->d, a->dtype, (uint64_t)out->d_cols, (uint64_t)a->m, (uint64_t)a->ldd * 2, 32, 32, 64);
  if (rc) return rc;
  out->tma_store = 1;
  if (a->residual && !a->swiglu && tma_res_enabled() && out->d_cols % 32 == 0 && ep.tail_begin >= n_out) {
    rc = make_tmap_2d_sw(tr, a->residual, a->dtype, (uint64_t)out->d_cols, (uint64_t)a->m, (uint64_t)a->ld_res * 2, 32,
                         32, 64);
    if (rc) return rc;
    out->res_tma = 1;
  }
  return TH_OK;
}

template <typename T, int BN, int EPI>
static int launch_tc(const th_gemm_args* a, const EpiParams& ep0, cudaStream_t st) {
  using C = TcCfg<BN>;
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, a->a, a->dtype, (uint64_t)a->k, (uint64_t)a->m, (uint64_t)a->lda * 2, 64, C::BM, true);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, a->w, a->dtype, (uint64_t)a->k, (uint64_t)a->n, (uint64_t)a->ldw * 2, 64, BN, true);
  if (rc) return rc;
  CUtensorMap td, tr;
  EpiParams ep;
  if ((rc = with_out_map(a, ep0, &ep, &td, &tr))) return rc;
  if ((rc = smem_limit(gemm_tc_kernel<T, BN, EPI>, C::SMEM_BYTES, "th_gemm(tcgen05)"))) return rc;
  const int tiles_m = (int)((a->m + C::BM - 1) / C::BM), tiles_n = (int)((a->n + BN - 1) / BN);
  const int ntiles = tiles_m * tiles_n;
  const int grid = ntiles < gemm_sms(a) ? ntiles : gemm_sms(a);
  // a GEMM kept to part of the GPU launches without PDL, so the SMs it leaves free stay free for the
  // kernel beside it (with PDL its CTAs would take them early, waiting for the previous kernel)
  launch_maybe_pdl(a->sm_limit <= 0, gemm_tc_kernel<T, BN, EPI>, dim3(grid), dim3(320), C::SMEM_BYTES, st, ta, tb, td,
                   tr, ep, (int)a->k, tiles_m, tiles_n);
  return check_launch("th_gemm(tcgen05)");
}

template <typename T, int BN, int EPI>
static int launch_tc2(const th_gemm_args* a, const EpiParams& ep0, cudaStream_t st) {
  using C = Tc2Cfg<BN>;
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, a->a, a->dtype, (uint64_t)a->k, (uint64_t)a->m, (uint64_t)a->lda * 2, 64, C::BM, true);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, a->w, a->dtype, (uint64_t)a->k, (uint64_t)a->n, (uint64_t)a->ldw * 2, 64, BN / 2, true);
  if (rc) return rc;
  CUtensorMap td, tr;
  EpiParams ep;
  if ((rc = with_out_map(a, ep0, &ep, &td, &tr))) return rc;
  if ((rc = smem_limit(gemm_tc2_kernel<T, BN, EPI>, C::SMEM_BYTES, "th_gemm(tcgen05 pair)"))) return rc;
  const int tiles_m = (int)((a->m + 2 * C::BM - 1) / (2 * C::BM)), tiles_n = (int)((a->n + BN - 1) / BN);
  const int ntiles = tiles_m * tiles_n, pairs = gemm_sms(a) / 2;
  const int grid = 2 * (ntiles < pairs ? ntiles : pairs);
  launch_maybe_pdl(a->sm_limit <= 0, gemm_tc2_kernel<T, BN, EPI>, dim3(grid), dim3(320), C::SMEM_BYTES, st, ta, tb,
                   td, tr, ep, (int)a->k, tiles_m, tiles_n);
  return check_launch("th_gemm(tcgen05 pair)");
}

// Tile width of the pair kernel: the one with the least wave-quantised work,
// rounds x (BN + 320).  The 320 is fitted to B200 timings: a tile costs far
// more than its width suggests at narrow widths (32768 x 3584 x 4096: 1071 /
// 778 / 660 us at BN 128 / 192 / 256, i.e. 49 / 33 / 25 rounds; 8192 x 3352 x
// 768: 69.6 / 53.3 / 49.2 us), so 256 wins unless it leaves a whole round
// nearly empty (8192 x 768 x 1536: 192 at 30.7 us against 31.6).  192 is
// offered only where no 64-column group (SwiGLU block, RoPE head,
// sum-of-squares group) may straddle the epilogue's column halves.
static int pair_mode() {  // TH_GEMM_PAIR: 0 single-CTA kernel, 1 (default) pair kernel, 128/192/256 its width
  static const int env = [] {
    const char* e = getenv("TH_GEMM_PAIR");
    return e ? atoi(e) : 1;
  }();
  return env;
}

static int pair_width(const th_gemm_args* a) {
  const int64_t tm = (a->m + 255) / 256, pairs = gemm_sms(a) / 2;
  const bool no192 = a->swiglu || a->rope_cos || a->ss_out;
  const int forced = pair_mode();
  if (forced == 256 || forced == 128 || (forced == 192 && !no192)) return forced;
  int best = 256;
  int64_t best_cost = INT64_MAX;
  for (int bn : {256, 192, 128}) {
    if (bn == 192 && no192) continue;
    const int64_t rounds = (tm * ((a->n + bn - 1) / bn) + pairs - 1) / pairs;
    const int64_t cost = rounds * (bn + 320);
    if (cost < best_cost) best_cost = cost, best = bn;
  }
  return best;
}

template <typename T>
static int dispatch_tc2(const th_gemm_args* a, const EpiParams& ep, cudaStream_t st) {
  const int bn = pair_width(a);
  if (a->swiglu) return bn == 256 ? launch_tc2<T, 256, EPI_SWIGLU>(a, ep, st) : launch_tc2<T, 128, EPI_SWIGLU>(a, ep, st);
  if (a->rope_cos) return bn == 256 ? launch_tc2<T, 256, EPI_ROPE>(a, ep, st) : launch_tc2<T, 128, EPI_ROPE>(a, ep, st);
  if (a->residual) {
    if (bn == 256) return launch_tc2<T, 256, EPI_RES>(a, ep, st);
    return bn == 192 ? launch_tc2<T, 192, EPI_RES>(a, ep, st) : launch_tc2<T, 128, EPI_RES>(a, ep, st);
  }
  if (bn == 256) return launch_tc2<T, 256, 0>(a, ep, st);
  return bn == 192 ? launch_tc2<T, 192, 0>(a, ep, st) : launch_tc2<T, 128, 0>(a, ep, st);
}

// The pair kernel serves every 2-byte GEMM with more than one 128-row tile
// (TH_GEMM_PAIR=0 in the environment selects the single-CTA kernel instead).
static bool use_pair(const th_gemm_args* a) { return pair_mode() != 0 && a->m > 128 && gemm_sms(a) >= 2; }

static bool is_al16(const void* p) { return p == nullptr || aligned16(p); }

template <typename T>
static int dispatch_tc(const th_gemm_args* a, const EpiParams& ep, cudaStream_t st, bool wide) {
  if (a->swiglu)
    return wide ? launch_tc<T, 256, EPI_SWIGLU>(a, ep, st) : launch_tc<T, 128, EPI_SWIGLU>(a, ep, st);
  if (a->rope_cos) return wide ? launch_tc<T, 256, EPI_ROPE>(a, ep, st) : launch_tc<T, 128, EPI_ROPE>(a, ep, st);
  if (a->residual) return wide ? launch_tc<T, 256, EPI_RES>(a, ep, st) : launch_tc<T, 128, EPI_RES>(a, ep, st);
  return wide ? launch_tc<T, 256, 0>(a, ep, st) : launch_tc<T, 128, 0>(a, ep, st);
}

}  // namespace th

extern "C" int th_gemm(const th_gemm_args* a, void* stream) {
  using namespace th;
  if (!a) return fail(TH_EINVAL, "th_gemm: args is NULL");
  if (!a->a || !a->w) return fail(TH_EINVAL, "th_gemm: a/w must be non-NULL");
  if (a->m <= 0 || a->n <= 0 || a->k <= 0) return fail(TH_EINVAL, "th_gemm: bad shape m=%lld n=%lld k=%lld", (long long)a->m, (long long)a->n, (long long)a->k);
  if (a->m > INT32_MAX || a->n > INT32_MAX || a->k > INT32_MAX) return fail(TH_EINVAL, "th_gemm: extent exceeds int32");
  if (a->dtype != TH_F32 && a->dtype != TH_BF16 && a->dtype != TH_F16) return fail(TH_EDTYPE, "th_gemm: unknown dtype %d", a->dtype);
  if (a->lda < a->k || a->ldw < a->k) return fail(TH_EINVAL, "th_gemm: lda/ldw smaller than k");
  const int64_t n_out = a->swiglu ? a->n / 2 : a->n;
  if (a->swiglu && a->n % 128) return fail(TH_EINVAL, "th_gemm: swiglu needs n %% 128 == 0 (64 gate | 64 up blocks)");
  if (n_out % 8) return fail(TH_EALIGN, "th_gemm: output width %lld must be a multiple of 8", (long long)n_out);
  // with out2, columns >= tail_begin are the fp32 tail (tail_begin 0: the whole output, d unused)
  const int tail = (a->out2 && a->tail_begin >= 0 && a->tail_begin < n_out) ? a->tail_begin : (int)n_out;
  if (tail % 8) return fail(TH_EALIGN, "th_gemm: tail_begin must be a multiple of 8");
  if (tail > 0 && !a->d) return fail(TH_EINVAL, "th_gemm: d must be non-NULL");
  if (tail > 0 && (a->ldd < tail || a->ldd % 8 || !is_al16(a->d)))
    return fail(TH_EALIGN, "th_gemm: d must be 16-B aligned with ldd %% 8 == 0 and ldd >= width");
  if (a->residual && (a->ld_res % 8 || !is_al16(a->residual))) return fail(TH_EALIGN, "th_gemm: residual must be 16-B aligned with ld_res %% 8 == 0");
  if (a->rope_cos) {
    const int hd = a->rope_head_dim;
    if (!a->rope_sin || hd <= 0 || hd % 2 || hd > 128 || a->rope_begin % hd || a->rope_end % hd || a->rope_seq <= 0)
      return fail(TH_EINVAL, "th_gemm: bad rope segment");
  }
  if (a->act < TH_ACT_NONE || a->act > TH_ACT_GELU_TANH) return fail(TH_EINVAL, "th_gemm: bad act %d", a->act);
  if (a->rs_parts && a->rs_nparts <= 0) return fail(TH_EINVAL, "th_gemm: rs_nparts must be > 0");
  if (a->ss_out && a->ss_ld < (n_out + 63) / 64) return fail(TH_EINVAL, "th_gemm: ss_ld too small");

  EpiParams ep;
  ep.d = a->d; ep.ldd = a->ldd; ep.m = (int)a->m; ep.n = (int)a->n;
  ep.rs_parts = a->rs_parts; ep.rs_nparts = a->rs_nparts; ep.rs_inv_k = a->rs_inv_k; ep.rs_eps = a->rs_eps;
  ep.act = a->act; ep.act_begin = a->act_begin; ep.act_end = a->act_end; ep.bias = a->bias;
  ep.rope_cos = a->rope_cos; ep.rope_sin = a->rope_sin; ep.rope_begin = a->rope_begin; ep.rope_end = a->rope_end;
  ep.rope_hd = a->rope_head_dim; ep.rope_seq = a->rope_seq;
  ep.rope_vec = a->rope_cos && is_al16(a->rope_cos) && is_al16(a->rope_sin) && a->rope_head_dim % 4 == 0;
  ep.rs_vec = a->rs_parts && is_al16(a->rs_parts) && a->rs_nparts % 4 == 0;
  ep.swiglu = a->swiglu; ep.residual = a->residual; ep.ld_res = a->ld_res;
  ep.out2 = a->out2; ep.ld_out2 = a->ld_out2; ep.tail_begin = tail;
  ep.ss_out = a->ss_out; ep.ss_ld = a->ss_ld;
  ep.tma_store = 0; ep.d_cols = tail; ep.res_tma = 0;  // the tcgen05 launchers set up the staged store
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

  if (a->dtype == TH_F32) {
    if (a->rope_cos && 128 % a->rope_head_dim) return fail(TH_EINVAL, "th_gemm: rope head_dim must divide 128");
    dim3 grid((unsigned)((a->n + SM_BN - 1) / SM_BN), (unsigned)((a->m + SM_BM - 1) / SM_BM));
    gemm_simt_kernel<float><<<grid, 256, 0, st>>>(reinterpret_cast<const float*>(a->a), a->lda,
                                                  reinterpret_cast<const float*>(a->w), a->ldw, ep, (int)a->k);
    return check_launch("th_gemm(fp32)");
  }
  // tcgen05 path: TMA wants 16-B aligned bases and row strides
  if (!aligned16(a->a) || !aligned16(a->w) || a->lda % 8 || a->ldw % 8)
    return fail(TH_EALIGN, "th_gemm: a/w must be 16-B aligned with lda, ldw multiples of 8");
  bool wide = a->n >= 256 && (!a->rope_cos || 256 % a->rope_head_dim == 0);
  if (wide) {  // narrow tiles when they cut the wave-quantised work by a fifth or more
    const int64_t tm = (a->m + 127) / 128, sms = gemm_sms(a);
    const int64_t r256 = (tm * ((a->n + 255) / 256) + sms - 1) / sms, r128 = (tm * ((a->n + 127) / 128) + sms - 1) / sms;
    if (r128 * 128 * 5 <= r256 * 256 * 4) wide = false;
  }
  if (use_pair(a)) {
    if (a->dtype == TH_BF16) return dispatch_tc2<__nv_bfloat16>(a, ep, st);
    return dispatch_tc2<__half>(a, ep, st);
  }
  if (a->dtype == TH_BF16) return dispatch_tc<__nv_bfloat16>(a, ep, st, wide);
  return dispatch_tc<__half>(a, ep, st, wide);
}
