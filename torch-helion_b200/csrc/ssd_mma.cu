// Tensor-core SSD passes for 2-byte inputs (bf16 / fp16), fp32 state.
//
// Same three-pass decomposition as ssd.cu (models/mamba.py:163-223); the two
// matrix-shaped passes run on m16n8k16 MMA tiles with fp32 accumulation:
//
//   state pass  states[p, n] = sum_l (x[l,p] w_l) B[l,n],  w_l = dt_l exp(cumA_last - cumA_l)
//               M = head_dim (16-row warp tiles), N = state columns, K = chunk rows
//   scan pass   per 64-row block i of a chunk:
//               y  = exp(cumA_i) * (C_i . S_in)                         (K = state)
//               G  = (C_i . B_j) * exp(cumA_i - cumA_j) * dt_j, j <= i  (K = state)
//               y += G . x_j                                            (K = rows j)
//               then D skip, silu(z) gate, store, per-head sum of squares.
// G never leaves registers: the fp32 accumulator fragment of one product is
// repacked as the bf16 A fragment of the next.  Operands are staged in
// shared memory with a 16-byte row pad so ldmatrix rows hit distinct banks.
#include "common.cuh"

namespace th {
namespace mma {

// pack2<T> (two values rounded and packed, `lo` low) comes from common.cuh

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

template <typename T> __device__ __forceinline__ void mma16816(float* d, const uint32_t* a, const uint32_t* b);
template <> __device__ __forceinline__ void mma16816<__nv_bfloat16>(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
template <> __device__ __forceinline__ void mma16816<__half>(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Lane addresses for ldmatrix.x4 (lane l: matrix l/8, row l%8 of it).
//  A row-major S[m][k]      (16x16 at m0,k0):  row m0+i+8*(mat&1), col k0+8*(mat>>1)
//  A stored S[k][m], .trans (16x16 at m0,k0):  row k0+i+8*(mat>>1), col m0+8*(mat&1)
//  B stored S[n][k]         (k16 x 2 n-tiles):  row n0+i+8*(mat>>1), col k0+8*(mat&1)
//  B stored S[k][n], .trans (k16 x 2 n-tiles):  row k0+i+8*(mat&1),  col n0+8*(mat>>1)
__device__ __forceinline__ uint32_t a_rowmajor(uint32_t base, int ld, int m0, int k0, int lane) {
  const int mat = lane >> 3, i = lane & 7;
  return base + (uint32_t)(((m0 + i + 8 * (mat & 1)) * ld + k0 + 8 * (mat >> 1)) * 2);
}
__device__ __forceinline__ uint32_t a_kmajor_t(uint32_t base, int ld, int m0, int k0, int lane) {
  const int mat = lane >> 3, i = lane & 7;
  return base + (uint32_t)(((k0 + i + 8 * (mat >> 1)) * ld + m0 + 8 * (mat & 1)) * 2);
}
__device__ __forceinline__ uint32_t b_nmajor(uint32_t base, int ld, int n0, int k0, int lane) {
  const int mat = lane >> 3, i = lane & 7;
  return base + (uint32_t)(((n0 + i + 8 * (mat >> 1)) * ld + k0 + 8 * (mat & 1)) * 2);
}
__device__ __forceinline__ uint32_t b_kmajor_t(uint32_t base, int ld, int n0, int k0, int lane) {
  const int mat = lane >> 3, i = lane & 7;
  return base + (uint32_t)(((k0 + i + 8 * (mat & 1)) * ld + n0 + 8 * (mat >> 1)) * 2);
}

// Asynchronous 16-byte global->shared copies (zero-filled when !valid).
__device__ __forceinline__ void cp_async16(void* sdst, const void* gsrc, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(sdst)), "l"(gsrc), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Asynchronous version of stage_rows (same layout, rows >= valid zero-filled).
template <typename T>
__device__ __forceinline__ void stage_rows_async(T* s, int lds, const T* g, int64_t ldg, int nrows, int ncols,
                                                 int valid, int tid, int nthreads) {
  const int vpr = ncols / 8;
  for (int v = tid; v < nrows * vpr; v += nthreads) {
    const int r = v / vpr, c = (v % vpr) * 8;
    const bool ok = r < valid;
    cp_async16(s + r * lds + c, ok ? (const void*)(g + (int64_t)r * ldg + c) : (const void*)g, ok);
  }
}

// Copy rows [r0, r0+nrows) x cols [0, ncols) of a strided global matrix into
// smem (row stride lds elements), zero-filling rows >= valid.  16-B vectors.
template <typename T>
__device__ __forceinline__ void stage_rows(T* s, int lds, const T* g, int64_t ldg, int nrows, int ncols, int valid,
                                           int tid, int nthreads) {
  const int vpr = ncols / 8;
  for (int v = tid; v < nrows * vpr; v += nthreads) {
    const int r = v / vpr, c = (v % vpr) * 8;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < valid) val = *reinterpret_cast<const uint4*>(g + (int64_t)r * ldg + c);
    *reinterpret_cast<uint4*>(s + r * lds + c) = val;
  }
}

}  // namespace mma

constexpr int MS_L = 256;   // max chunk
constexpr int MS_LH = 128;  // state pass: rows staged at a time
constexpr int MS_NS = 128;  // state pass: state columns per CTA
constexpr int MS_RB = 64;   // scan pass: rows per CTA

struct MmaGeom {
  int batch, seq, heads, hd, groups, ns, chunk, nchunks, nsplit;
};

__host__ __device__ inline int64_t mg_cum(const MmaGeom& g, int b, int h, int c, int l) {
  return (((int64_t)b * g.heads + h) * g.nchunks + c) * g.chunk + l;
}

// ------------------------------------------------------------ state pass
// grid (nchunks, heads, batch*nsplit), 256 threads.  P = head_dim.
template <typename T, int P>
__global__ void __launch_bounds__(256) ssd_state_mma(th_ssd_args p, MmaGeom g, float* __restrict__ states,
                                                     float* __restrict__ cum) {
  using namespace mma;
  extern __shared__ __align__(16) uint8_t smraw[];
  constexpr int LDX = P + 8, LDB = MS_NS + 8;
  float* w = reinterpret_cast<float*>(smraw);                  // [MS_L]
  T* xs = reinterpret_cast<T*>(w + MS_L);                      // [MS_LH][LDX]
  T* bs = xs + MS_LH * LDX;                                    // [MS_LH][LDB]
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z / g.nsplit, split = blockIdx.z % g.nsplit;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hg = h / (g.heads / g.groups);
  const int s0 = c * g.chunk, len = min(g.chunk, g.seq - s0);
  const int64_t t0 = (int64_t)b * g.seq + s0;
  const int n_base = split * MS_NS, ncols = min(MS_NS, g.ns - n_base);
  // in-chunk cumsum of dt*A (Hillis-Steele over <= 256 rows)
  const float A = p.A[h];
  float dtv = 0.f, v = 0.f;
  if (tid < g.chunk) {
    dtv = tid < len ? p.dt[(t0 + tid) * p.lddt + h] : 0.f;
    v = dtv * A;
    w[tid] = v;
  }
  __syncthreads();
  for (int off = 1; off < g.chunk; off <<= 1) {
    float add = (tid < g.chunk && tid >= off) ? w[tid - off] : 0.f;
    __syncthreads();
    if (tid < g.chunk) { v += add; w[tid] = v; }
    __syncthreads();
  }
  const float last = w[len - 1];
  __syncthreads();
  if (tid < g.chunk) {
    if (split == 0) cum[mg_cum(g, b, h, c, tid)] = v;
    w[tid] = tid < len ? dtv * __expf(last - v) : 0.f;
  }
  __syncthreads();
  // warp tiling of the [P x ncols] output: MT m-tiles, the rest split N
  constexpr int MT = P / 16;
  constexpr int NGRP = 8 / MT;                  // warps sharing an m-tile
  constexpr int NT = (MS_NS / 8) / NGRP;        // n-tiles per warp (max)
  const int mt = warp % MT, ng = warp / MT;
  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  const T* xg = reinterpret_cast<const T*>(p.x) + (int64_t)h * P;
  const T* bg = reinterpret_cast<const T*>(p.B) + (int64_t)hg * g.ns + n_base;
  const uint32_t xs_a = smem_u32(xs), bs_a = smem_u32(bs);
  for (int l0 = 0; l0 < len; l0 += MS_LH) {
    const int rows = min(MS_LH, len - l0);
    // x rows scaled by w, rounded to T
    for (int e = tid; e < MS_LH * (P / 8); e += 256) {
      const int r = e / (P / 8), cc = (e % (P / 8)) * 8;
      float f[8];
      if (r < rows) {
        load8<T>(xg + (t0 + l0 + r) * p.ldx + cc, f);
        const float wr = w[l0 + r];
#pragma unroll
        for (int q = 0; q < 8; ++q) f[q] *= wr;
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) f[q] = 0.f;
      }
      store8<T>(xs + r * LDX + cc, f);
    }
    stage_rows_async<T>(bs, LDB, bg + (t0 + l0) * p.ldb, p.ldb, MS_LH, ncols, rows, tid, 256);
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    const int kmax = (rows + 15) / 16;
    for (int kk = 0; kk < kmax; ++kk) {
      uint32_t a[4];
      ldsm_x4_t(a_kmajor_t(xs_a, LDX, mt * 16, kk * 16, lane), a);
#pragma unroll
      for (int j = 0; j < NT; j += 2) {
        const int n0 = (ng * NT + j) * 8;
        if (n0 < ncols) {
          uint32_t bb[4];
          ldsm_x4_t(b_kmajor_t(bs_a, LDB, n0, kk * 16, lane), bb);
          mma16816<T>(acc[j], a, bb);
          mma16816<T>(acc[j + 1], a, bb + 2);
        }
      }
    }
    __syncthreads();
  }
  float* dst = states + (((int64_t)b * g.nchunks + c) * g.heads + h) * (int64_t)(P * g.ns) + n_base;
  const int gr = lane >> 2, tq = lane & 3;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int n = (ng * NT + j) * 8 + tq * 2;
    if (n < ncols) {
      const int r0 = mt * 16 + gr;
      *reinterpret_cast<float2*>(dst + (int64_t)r0 * g.ns + n) = make_float2(acc[j][0], acc[j][1]);
      *reinterpret_cast<float2*>(dst + (int64_t)(r0 + 8) * g.ns + n) = make_float2(acc[j][2], acc[j][3]);
    }
  }
}

// ------------------------------------------------------------- scan pass
// grid (nchunks * chunk/64, heads, batch), 128 threads (4 warps x 16 rows).
// C rows and S_in are staged once; the (B, x) blocks of the intra-chunk
// loop are double-buffered with cp.async so block j+1 loads while block j
// multiplies.  S_in stays fp32 in shared memory and its MMA fragments are
// packed straight from it.
template <typename T, int P>
__global__ void __launch_bounds__(128) ssd_scan_mma(th_ssd_args p, MmaGeom g, const float* __restrict__ states,
                                                    const float* __restrict__ cum) {
  using namespace mma;
  extern __shared__ __align__(16) uint8_t smraw[];
  const int LDN = g.ns + 8;       // bf16 row stride of C/B tiles
  const int LDS = g.ns + 4;       // fp32 row stride of the S_in tile
  constexpr int LDP = P + 8;
  T* Cs = reinterpret_cast<T*>(smraw);                              // [64][LDN]
  float* Sf = reinterpret_cast<float*>(Cs + MS_RB * LDN);           // [P][LDS]
  T* Bs = reinterpret_cast<T*>(Sf + P * LDS);                       // [2][64][LDN]
  T* xs = Bs + 2 * MS_RB * LDN;                                     // [2][64][LDP]
  float* ci = reinterpret_cast<float*>(xs + 2 * MS_RB * LDP);       // [64]
  float* cj = ci + MS_RB;                                           // [2][64]
  float* dj = cj + 2 * MS_RB;                                       // [2][64]
  const int rb_per = g.chunk / MS_RB;
  const int c = blockIdx.x / rb_per, rb = blockIdx.x % rb_per;
  const int h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gr = lane >> 2, tq = lane & 3;
  const int hg = h / (g.heads / g.groups);
  const int s0 = c * g.chunk, len = min(g.chunk, g.seq - s0);
  const int i0 = rb * MS_RB;
  if (i0 >= len) return;
  const int64_t t0 = (int64_t)b * g.seq + s0;
  const T* xg = reinterpret_cast<const T*>(p.x) + (int64_t)h * P;
  const T* Bg = reinterpret_cast<const T*>(p.B) + (int64_t)hg * g.ns;
  const T* Cg = reinterpret_cast<const T*>(p.C) + (int64_t)hg * g.ns;
  const float* Sin = states + (((int64_t)b * g.nchunks + c) * g.heads + h) * (int64_t)(P * g.ns);
  const int nj = i0 / MS_RB + 1;  // intra-chunk blocks j0 = 0 .. i0

  auto stage_j = [&](int jb, int buf) {
    const int j0 = jb * MS_RB;
    stage_rows_async<T>(Bs + buf * MS_RB * LDN, LDN, Bg + (t0 + j0) * p.ldb, p.ldb, MS_RB, g.ns, len - j0, tid, 128);
    stage_rows_async<T>(xs + buf * MS_RB * LDP, LDP, xg + (t0 + j0) * p.ldx, p.ldx, MS_RB, P, len - j0, tid, 128);
    if (tid < MS_RB) {
      const bool ok = j0 + tid < len;
      cj[buf * MS_RB + tid] = ok ? cum[mg_cum(g, b, h, c, j0 + tid)] : 0.f;
      dj[buf * MS_RB + tid] = ok ? p.dt[(t0 + j0 + tid) * p.lddt + h] : 0.f;
    }
  };
  // group 0: C rows + S_in ; group 1: first (B, x) block
  stage_rows_async<T>(Cs, LDN, Cg + (t0 + i0) * p.ldc, p.ldc, MS_RB, g.ns, len - i0, tid, 128);
  for (int v = tid; v < P * (g.ns / 4); v += 128) {
    const int r = v / (g.ns / 4), cc = (v % (g.ns / 4)) * 4;
    cp_async16(Sf + r * LDS + cc, Sin + (int64_t)r * g.ns + cc, true);
  }
  if (tid < MS_RB) ci[tid] = (i0 + tid < len) ? cum[mg_cum(g, b, h, c, i0 + tid)] : 0.f;
  cp_async_commit();
  stage_j(0, 0);
  cp_async_commit();
  cp_async_wait<1>();
  __syncthreads();

  const uint32_t Cs_a = smem_u32(Cs);
  constexpr int PT = P / 8;  // n-tiles of y
  float y[PT][4];
#pragma unroll
  for (int j = 0; j < PT; ++j) y[j][0] = y[j][1] = y[j][2] = y[j][3] = 0.f;
  // y_off = C . S_in^T : B fragment (k = state n, col = p) packed from fp32 S[p][n]
  for (int kk = 0; kk < g.ns / 16; ++kk) {
    uint32_t a[4];
    ldsm_x4(a_rowmajor(Cs_a, LDN, warp * 16, kk * 16, lane), a);
#pragma unroll
    for (int j = 0; j < PT; ++j) {
      const float* sp = Sf + (j * 8 + gr) * LDS + kk * 16 + tq * 2;
      const float2 lo = *reinterpret_cast<const float2*>(sp);
      const float2 hi = *reinterpret_cast<const float2*>(sp + 8);
      uint32_t bb[2] = {pack2<T>(lo.x, lo.y), pack2<T>(hi.x, hi.y)};
      mma16816<T>(y[j], a, bb);
    }
  }
  const int rA = warp * 16 + gr, rB = rA + 8;
  const float ciA = ci[rA], ciB = ci[rB];
  const float eA = __expf(ciA), eB = __expf(ciB);
#pragma unroll
  for (int j = 0; j < PT; ++j) {
    y[j][0] *= eA; y[j][1] *= eA; y[j][2] *= eB; y[j][3] *= eB;
  }
  const int giA = i0 + rA, giB = i0 + rB;
  for (int jb = 0; jb < nj; ++jb) {
    const int buf = jb & 1;
    if (jb + 1 < nj) stage_j(jb + 1, buf ^ 1);  // prefetch the next block
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t Bs_a = smem_u32(Bs + buf * MS_RB * LDN), xs_a = smem_u32(xs + buf * MS_RB * LDP);
    const float* cjb = cj + buf * MS_RB;
    const float* djb = dj + buf * MS_RB;
    const int j0 = jb * MS_RB;
    float G[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) G[j][0] = G[j][1] = G[j][2] = G[j][3] = 0.f;
    for (int kk = 0; kk < g.ns / 16; ++kk) {
      uint32_t a[4];
      ldsm_x4(a_rowmajor(Cs_a, LDN, warp * 16, kk * 16, lane), a);
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        uint32_t bb[4];
        ldsm_x4(b_nmajor(Bs_a, LDN, j * 8, kk * 16, lane), bb);
        mma16816<T>(G[j], a, bb);
        mma16816<T>(G[j + 1], a, bb + 2);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int jl = j * 8 + tq * 2 + q, gj = j0 + jl;
        const float wj = djb[jl], cjv = cjb[jl];
        G[j][q] = (gj <= giA) ? G[j][q] * __expf(ciA - cjv) * wj : 0.f;
        G[j][2 + q] = (gj <= giB) ? G[j][2 + q] * __expf(ciB - cjv) * wj : 0.f;
      }
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      a[0] = pack2<T>(G[2 * kk][0], G[2 * kk][1]);
      a[1] = pack2<T>(G[2 * kk][2], G[2 * kk][3]);
      a[2] = pack2<T>(G[2 * kk + 1][0], G[2 * kk + 1][1]);
      a[3] = pack2<T>(G[2 * kk + 1][2], G[2 * kk + 1][3]);
#pragma unroll
      for (int j = 0; j < PT; j += 2) {
        uint32_t bb[4];
        ldsm_x4_t(b_kmajor_t(xs_a, LDP, j * 8, kk * 16, lane), bb);
        mma16816<T>(y[j], a, bb);
        mma16816<T>(y[j + 1], a, bb + 2);
      }
    }
    __syncthreads();  // buffer `buf` is refilled two iterations later
  }
  // epilogue: D skip (x of the diagonal block is still staged), gate, store,
  // per-head sum of squares
  const T* xd = xs + ((nj - 1) & 1) * MS_RB * LDP;
  const float Dh = p.D ? p.D[h] : 0.f;
  const T* zg = reinterpret_cast<const T*>(p.z);
  T* out = reinterpret_cast<T*>(p.out);
  float ssA = 0.f, ssB = 0.f;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int rl = half ? rB : rA;
    const int gi = i0 + rl;
    if (gi >= len) continue;
    const int64_t t = t0 + gi;
#pragma unroll
    for (int j = 0; j < PT; ++j) {
      const int col = j * 8 + tq * 2;
      float v0 = y[j][2 * half] + Dh * to_f32(xd[rl * LDP + col]);
      float v1 = y[j][2 * half + 1] + Dh * to_f32(xd[rl * LDP + col + 1]);
      if (zg) {
        const uint32_t zz = *reinterpret_cast<const uint32_t*>(zg + t * p.ldz + (int64_t)h * P + col);
        const T* zp = reinterpret_cast<const T*>(&zz);
        v0 *= silu_f(to_f32(zp[0]));
        v1 *= silu_f(to_f32(zp[1]));
      }
      *reinterpret_cast<uint32_t*>(out + t * p.ldo + (int64_t)h * P + col) = pack2<T>(v0, v1);
      const float q0 = round_to<T>(v0), q1 = round_to<T>(v1);
      if (half) ssB += q0 * q0 + q1 * q1; else ssA += q0 * q0 + q1 * q1;
    }
  }
  ssA += __shfl_xor_sync(0xffffffffu, ssA, 1);
  ssA += __shfl_xor_sync(0xffffffffu, ssA, 2);
  ssB += __shfl_xor_sync(0xffffffffu, ssB, 1);
  ssB += __shfl_xor_sync(0xffffffffu, ssB, 2);
  if (p.gss && tq == 0) {
    if (giA < len) p.gss[(t0 + giA) * p.ldgss + h] = ssA;
    if (giB < len) p.gss[(t0 + giB) * p.ldgss + h] = ssB;
  }
}

// The inter-chunk pass is shared with the fp32 path (ssd.cu: ssd_pass_kernel).

}  // namespace th

#include "ssd_tc.cu"  // tcgen05 scan pass (head_dim 64, chunk 256)

namespace th {

template <typename T, int P>
static int ssd_mma_launch(const th_ssd_args* a, const MmaGeom& g, float* states, float* cum, cudaStream_t st) {
  const size_t sm1 = sizeof(float) * MS_L + sizeof(T) * (MS_LH * (P + 8) + MS_LH * (MS_NS + 8));
  const size_t sm3 = sizeof(T) * (3 * MS_RB * (g.ns + 8) + 2 * MS_RB * (P + 8)) + sizeof(float) * (P * (g.ns + 4) + 5 * MS_RB);
  if (int rc = smem_limit(ssd_state_mma<T, P>, sm1, "th_ssd(state, mma)")) return rc;
  if (int rc = smem_limit(ssd_scan_mma<T, P>, sm3, "th_ssd(scan, mma)")) return rc;
  ssd_state_mma<T, P><<<dim3(g.nchunks, g.heads, g.batch * g.nsplit), 256, sm1, st>>>(*a, g, states, cum);
  int rc = check_launch("th_ssd(state, mma)");
  if (rc) return rc;
  SsdGeom sg{g.batch, g.seq, g.heads, g.hd, g.groups, g.ns, g.chunk, g.nchunks,
             (int64_t)g.batch * g.nchunks * g.heads * g.hd * g.ns};
  ssd_pass_kernel<<<dim3((g.hd * g.ns + 255) / 256, g.heads, g.batch), 256, 0, st>>>(sg, states, cum);
  rc = check_launch("th_ssd(pass)");
  if (rc) return rc;
  if (P == TS_P && ssd_scan_tc_try<T>(a, g.nchunks, states, cum, st, &rc) == 0) return rc;
  ssd_scan_mma<T, P><<<dim3(g.nchunks * (g.chunk / MS_RB), g.heads, g.batch), 128, sm3, st>>>(*a, g, states, cum);
  return check_launch("th_ssd(scan, mma)");
}

// Tensor-core path applies to 2-byte dtypes with head_dim in {16, 32, 64},
// state_dim a multiple of 16 (<= 256), chunk a multiple of 64, and 16-byte
// aligned rows.  Returns 1 (not taken) when the shape is outside that set.
template <typename T>
static int ssd_mma_try(const th_ssd_args* a, float* states, float* cum, cudaStream_t st, int* rc) {
  const int P = a->head_dim, N = a->state_dim;
  if (N % 16 || N > 256 || a->chunk % MS_RB || a->chunk > MS_L) return 1;
  if (P != 16 && P != 32 && P != 64) return 1;
  auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!al(a->x) || !al(a->B) || !al(a->C) || a->ldx % 8 || a->ldb % 8 || a->ldc % 8) return 1;
  if (a->z && ((reinterpret_cast<uintptr_t>(a->z) & 3) || a->ldz % 2)) return 1;
  MmaGeom g{a->batch, a->seq, a->heads, P, a->ngroups, N, a->chunk, (a->seq + a->chunk - 1) / a->chunk,
            (N + MS_NS - 1) / MS_NS};
  switch (P) {
    case 16: *rc = ssd_mma_launch<T, 16>(a, g, states, cum, st); break;
    case 32: *rc = ssd_mma_launch<T, 32>(a, g, states, cum, st); break;
    default: *rc = ssd_mma_launch<T, 64>(a, g, states, cum, st); break;
  }
  return 0;
}

}  // namespace th
