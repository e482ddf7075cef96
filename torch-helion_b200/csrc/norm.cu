// Memory-bound row kernels: RMSNorm statistics / standalone RMSNorm,
// depthwise causal conv1d + activation, embedding gather.
// One warp per row with 16-byte vector loads; grids sized in multiples of
// the SM count by the launchers.
#include "common.cuh"

namespace th {

// ------------------------------------------------------------- rowstat
// Rows of up to 32*8*RV elements (multiples of 8) are held in registers:
// every 16-byte load of a row is issued before the first one is used.  RV
// (16-byte vectors per lane) is 4 for rows up to 1024 elements, else 16.
template <typename T, int RV>
__global__ void __launch_bounds__(256) rowstat_kernel(const T* __restrict__ x, int64_t ldx, float* __restrict__ out,
                                                      int64_t rows, int cols) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = wid; r < rows; r += nw) {
    const T* p = x + r * ldx;
    float s = 0.f;
    if ((cols & 7) == 0 && cols <= 256 * RV) {
      uint4 u[RV];
#pragma unroll
      for (int k = 0; k < RV; ++k) {
        const int c = (k * 32 + lane) * 8;
        if (c < cols) u[k] = *reinterpret_cast<const uint4*>(p + c);
      }
#pragma unroll
      for (int k = 0; k < RV; ++k) {
        if ((k * 32 + lane) * 8 >= cols) break;
        const T* h = reinterpret_cast<const T*>(&u[k]);
#pragma unroll
        for (int e = 0; e < 16 / (int)sizeof(T); ++e) { const float v = to_f32(h[e]); s = fmaf(v, v, s); }
        if constexpr (sizeof(T) == 4) {  // fp32: the second half of the 8 elements
          const float4 b = *reinterpret_cast<const float4*>(p + (k * 32 + lane) * 8 + 4);
          s = fmaf(b.x, b.x, s); s = fmaf(b.y, b.y, s); s = fmaf(b.z, b.z, s); s = fmaf(b.w, b.w, s);
        }
      }
    } else if ((cols & 7) == 0) {
      for (int c = lane * 8; c < cols; c += 256) {
        float v[8];
        load8<T>(p + c, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) s = fmaf(v[e], v[e], s);
      }
    } else {
      for (int c = lane; c < cols; c += 32) {
        float v = to_f32(p[c]);
        s = fmaf(v, v, s);
      }
    }
    s = warp_sum(s);
    if (lane == 0) out[r] = s;
  }
}

// ------------------------------------------------------------- rmsnorm
template <typename T, int RV>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const T* __restrict__ x, int64_t ldx, const float* __restrict__ g,
                                                      T* __restrict__ y, int64_t ldy, int64_t rows, int cols, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = wid; r < rows; r += nw) {
    const T* p = x + r * ldx;
    T* q = y + r * ldy;
    float s = 0.f;
    if constexpr (sizeof(T) == 2) {
      if ((cols & 7) == 0 && cols <= 256 * RV) {  // one pass: the row stays in registers
        uint4 u[RV];
#pragma unroll
        for (int k = 0; k < RV; ++k) {
          const int c = (k * 32 + lane) * 8;
          if (c < cols) u[k] = *reinterpret_cast<const uint4*>(p + c);
        }
#pragma unroll
        for (int k = 0; k < RV; ++k) {
          if ((k * 32 + lane) * 8 >= cols) break;
          const T* h = reinterpret_cast<const T*>(&u[k]);
#pragma unroll
          for (int e = 0; e < 8; ++e) { const float v = to_f32(h[e]); s = fmaf(v, v, s); }
        }
        s = warp_sum(s);
        const float rs = rsqrtf(s / (float)cols + eps);
#pragma unroll
        for (int k = 0; k < RV; ++k) {
          const int c = (k * 32 + lane) * 8;
          if (c >= cols) break;
          const T* h = reinterpret_cast<const T*>(&u[k]);
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = to_f32(h[e]) * rs * (g ? g[c + e] : 1.f);
          store8<T>(q + c, v);
        }
        continue;
      }
    }
    const bool vec = (cols & 7) == 0;
    if (vec) {
      for (int c = lane * 8; c < cols; c += 256) {
        float v[8];
        load8<T>(p + c, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) s = fmaf(v[e], v[e], s);
      }
    } else {
      for (int c = lane; c < cols; c += 32) {
        float v = to_f32(p[c]);
        s = fmaf(v, v, s);
      }
    }
    s = warp_sum(s);
    const float rs = rsqrtf(s / (float)cols + eps);
    if (vec) {
      for (int c = lane * 8; c < cols; c += 256) {
        float v[8];
        load8<T>(p + c, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = v[e] * rs * (g ? g[c + e] : 1.f);
        store8<T>(q + c, v);
      }
    } else {
      for (int c = lane; c < cols; c += 32) q[c] = from_f32<T>(to_f32(p[c]) * rs * (g ? g[c] : 1.f));
    }
  }
}

// ------------------------------------------- 2-byte rows held in registers
// Rows of up to 256*RV elements (multiples of 8) of a 2-byte type: a warp
// issues every 16-byte load of ROWS rows before the first is used, so each
// warp keeps ROWS * cols * 2 bytes in flight.  The RMSNorm gain is staged in
// shared memory once per block (16-byte reads, no per-element global loads).
template <typename T, int RV, int ROWS>
__global__ void __launch_bounds__(256) rowstat_rows(const T* __restrict__ x, int64_t ldx, float* __restrict__ out,
                                                    int64_t rows, int cols) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r0 = wid * ROWS; r0 < rows; r0 += nw * ROWS) {
    uint4 u[ROWS][RV];
#pragma unroll
    for (int k = 0; k < RV; ++k) {
      const int c = (k * 32 + lane) * 8;
#pragma unroll
      for (int j = 0; j < ROWS; ++j)
        if (c < cols && r0 + j < rows) u[j][k] = *reinterpret_cast<const uint4*>(x + (r0 + j) * ldx + c);
    }
    float s[ROWS];
#pragma unroll
    for (int j = 0; j < ROWS; ++j) {
      s[j] = 0.f;
#pragma unroll
      for (int k = 0; k < RV; ++k) {
        if ((k * 32 + lane) * 8 >= cols) break;
        const T* h = reinterpret_cast<const T*>(&u[j][k]);
#pragma unroll
        for (int e = 0; e < 8; ++e) { const float v = to_f32(h[e]); s[j] = fmaf(v, v, s[j]); }
      }
      s[j] = warp_sum(s[j]);
    }
    if (lane == 0) {
#pragma unroll
      for (int j = 0; j < ROWS; ++j)
        if (r0 + j < rows) out[r0 + j] = s[j];
    }
  }
}

template <typename T, int RV, int ROWS>
__global__ void __launch_bounds__(256) rmsnorm_rows(const T* __restrict__ x, int64_t ldx, const float* __restrict__ g,
                                                    T* __restrict__ y, int64_t ldy, int64_t rows, int cols, float eps) {
  extern __shared__ float4 gain4[];  // cols / 4
  float* gain = reinterpret_cast<float*>(gain4);
  pdl_wait();
  pdl_trigger();
  for (int c = threadIdx.x; c < cols; c += blockDim.x) gain[c] = g ? g[c] : 1.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r0 = wid * ROWS; r0 < rows; r0 += nw * ROWS) {
    uint4 u[ROWS][RV];
#pragma unroll
    for (int k = 0; k < RV; ++k) {
      const int c = (k * 32 + lane) * 8;
#pragma unroll
      for (int j = 0; j < ROWS; ++j)
        if (c < cols && r0 + j < rows) u[j][k] = *reinterpret_cast<const uint4*>(x + (r0 + j) * ldx + c);
    }
#pragma unroll
    for (int j = 0; j < ROWS; ++j) {
      if (r0 + j >= rows) break;
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < RV; ++k) {
        if ((k * 32 + lane) * 8 >= cols) break;
        const T* h = reinterpret_cast<const T*>(&u[j][k]);
#pragma unroll
        for (int e = 0; e < 8; ++e) { const float v = to_f32(h[e]); s = fmaf(v, v, s); }
      }
      s = warp_sum(s);
      const float rs = rsqrtf(s / (float)cols + eps);
#pragma unroll
      for (int k = 0; k < RV; ++k) {
        const int c = (k * 32 + lane) * 8;
        if (c >= cols) break;
        const T* h = reinterpret_cast<const T*>(&u[j][k]);
        const float4 ga = gain4[c / 4], gb = gain4[c / 4 + 1];
        const float gv[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = to_f32(h[e]) * rs * gv[e];
        store8<T>(y + (r0 + j) * ldy + c, v);
      }
    }
  }
}

// ------------------------------------------------------ causal conv1d
// One thread = CONV_TPT consecutive tokens x 8 consecutive channels; a
// 32 x CONV_TY block covers 256 channels x (CONV_TY*CONV_TPT) tokens.  A warp reads 512
// contiguous bytes of a row; a thread keeps its CONV_TPT+width-1 input rows
// packed (16 bytes each) in registers, all issued before the first use, so
// the halo is re-read only width-1 times per CONV_TPT tokens and the weights
// (8 channels x width taps, float4 loads) once per CONV_TPT tokens.
constexpr int CONV_TPT = 8, CONV_TY = 4;  // tokens per thread, token groups per block

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float* v) {
  if constexpr (sizeof(T) == 2) {
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = to_f32(h[e]);
  }
}

template <typename T, int W>
__global__ void __launch_bounds__(128) conv1d_kernel(const T* __restrict__ x, int64_t ldx, const float* __restrict__ w,
                                                     const float* __restrict__ bias, T* __restrict__ y, int64_t ldy,
                                                     int batch, int seq, int channels, int act) {
  const int c0 = (blockIdx.x * 32 + threadIdx.x) * 8;
  const int64_t t0 = ((int64_t)blockIdx.y * CONV_TY + threadIdx.y) * CONV_TPT;  // first token (global row)
  const int64_t T_ = (int64_t)batch * seq;
  // the block's 256 x W weights, tap-major in shared memory (coalesced global
  // reads; a thread then reads its 8 channels of one tap as two float4)
  __shared__ __align__(16) float wsm[W][256];
  {
    const int cb = blockIdx.x * 256;
    for (int i = threadIdx.y * 32 + threadIdx.x; i < 256 * W; i += 32 * CONV_TY) {
      const int cl = i / W, j = i % W;
      wsm[j][cl] = cb + cl < channels ? w[(int64_t)(cb + cl) * W + j] : 0.f;
    }
  }
  __syncthreads();
  if (c0 >= channels || t0 >= T_) return;
  // global rows t0-(W-1) .. t0+CONV_TPT-1 (a thread's tokens may straddle two
  // sequences; taps that would reach into the previous sequence are masked)
  constexpr int R = CONV_TPT + W - 1;
  float wt[8][W];
  float bi[8];
  if constexpr (sizeof(T) == 2) {
    uint4 raw[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t tr = t0 - (W - 1) + r;
      raw[r] = (tr >= 0 && tr < T_) ? *reinterpret_cast<const uint4*>(x + tr * ldx + c0) : make_uint4(0, 0, 0, 0);
    }
    const int cl = threadIdx.x * 8;
#pragma unroll
    for (int j = 0; j < W; ++j) {
      const float4 a = *reinterpret_cast<const float4*>(&wsm[j][cl]);
      const float4 b = *reinterpret_cast<const float4*>(&wsm[j][cl + 4]);
      wt[0][j] = a.x; wt[1][j] = a.y; wt[2][j] = a.z; wt[3][j] = a.w;
      wt[4][j] = b.x; wt[5][j] = b.y; wt[6][j] = b.z; wt[7][j] = b.w;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) bi[e] = bias ? bias[c0 + e] : 0.f;
    float in[R][8];
#pragma unroll
    for (int r = 0; r < R; ++r) unpack8<T>(raw[r], in[r]);
    int sk = (int)(t0 % seq);  // position of token t0 in its sequence
#pragma unroll
    for (int k = 0; k < CONV_TPT; ++k, ++sk) {
      if (sk == seq) sk = 0;
      const int64_t t = t0 + k;
      if (t >= T_) break;
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = bi[e];
      if (sk >= W - 1) {
#pragma unroll
        for (int j = 0; j < W; ++j)
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] = fmaf(wt[e][j], in[k + j][e], o[e]);
      } else {
#pragma unroll
        for (int j = 0; j < W; ++j) {
          if (sk - (W - 1) + j < 0) continue;  // zero left padding of the causal conv
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] = fmaf(wt[e][j], in[k + j][e], o[e]);
        }
      }
      if (act == TH_ACT_SILU) {
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = silu_f(o[e]);
      }
      store8<T>(y + t * ldy + c0, o);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e)
#pragma unroll
      for (int j = 0; j < W; ++j) wt[e][j] = w[(int64_t)(c0 + e) * W + j];
#pragma unroll
    for (int e = 0; e < 8; ++e) bi[e] = bias ? bias[c0 + e] : 0.f;
    for (int k = 0; k < CONV_TPT; ++k) {
      const int64_t t = t0 + k;
      if (t >= T_) break;
      const int sk = (int)(t % seq);
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = bi[e];
      for (int j = 0; j < W; ++j) {
        const int64_t tr = t - (W - 1) + j;
        if (sk - (W - 1) + j < 0) continue;
        float in[8];
        load8<T>(x + tr * ldx + c0, in);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = fmaf(wt[e][j], in[e], o[e]);
      }
      if (act == TH_ACT_SILU) {
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = silu_f(o[e]);
      }
      store8<T>(y + t * ldy + c0, o);
    }
  }
}

// TMA-staged causal conv (2-byte dtypes): a persistent block streams tiles
// of 32 tokens x 256 channels through a 3-stage shared-memory ring.  Each
// tile is one TMA box of (32 + width - 1) rows starting width-1 rows before
// the tile; the 3-D map [batch][seq][channels] zero-fills rows before the
// sequence start, which is exactly the causal left padding, and rows past
// its end.  Thread = 8 channels x 4 tokens, read from shared memory
// conflict-free (a warp reads one 512-byte row).  The outputs go to one of two
// shared-memory output tiles and leave by TMA store, which clips rows past the
// sequence end and channels past the last one, so the threads issue no global
// stores (per-thread 16-byte stores of every output stalled on the LSU queue).
constexpr int CT_TOK = 32, CT_CH = 256, CT_STAGES = 3;

template <int W>
struct CtCfg {
  static constexpr int ROWS = CT_TOK + W - 1;
  static constexpr int TILE = ((ROWS * CT_CH * 2 + 127) / 128) * 128;
  static constexpr int OUT = CT_TOK * CT_CH * 2;  // one output tile
  static constexpr int OFF_OUT = CT_STAGES * TILE;
  static constexpr int OFF_W = OFF_OUT + 2 * OUT;        // taps of the block's channels, [W][CT_CH] fp32
  static constexpr int OFF_B = OFF_W + W * CT_CH * 4;    // bias, [CT_CH] fp32
  static constexpr int OFF_BAR = OFF_B + CT_CH * 4;
  static constexpr int SMEM = 128 + OFF_BAR + 64;
};

template <typename T, int W>
__global__ void __launch_bounds__(256, 2) conv1d_tma(const __grid_constant__ CUtensorMap tmX,
                                                     const __grid_constant__ CUtensorMap tmY, const float* __restrict__ w,
                                                     const float* __restrict__ bias, int channels, int act, int ncb,
                                                     int nsb, int ntiles) {
  using Cf = CtCfg<W>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_align<128>(smem_raw);
  uint8_t* outs = sm + Cf::OFF_OUT;  // [2] output tiles
  float* wsm = reinterpret_cast<float*>(sm + Cf::OFF_W);
  float* bsm = reinterpret_cast<float*>(sm + Cf::OFF_B);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + Cf::OFF_BAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bar + CT_STAGES);
  const int tid = threadIdx.x, tx = tid & 31, ty = tid >> 5;
  // gridDim.x is a multiple of ncb, so every tile of this block has the same channel block
  const int cb = blockIdx.x % ncb;
  auto coords = [&](int tile, int& sb, int& b) {
    const int rest = tile / ncb;
    sb = rest % nsb;
    b = rest / nsb;
  };
  auto issue = [&](int k) {  // k-th tile of this block into stage k % CT_STAGES
    const int tile = blockIdx.x + k * gridDim.x;
    if (tile >= ntiles) return;
    int sb, b;
    coords(tile, sb, b);
    uint64_t* br = &bar[k % CT_STAGES];
    mbar_arrive_expect_tx(br, Cf::ROWS * CT_CH * 2);
    tma_load_3d(sm + (k % CT_STAGES) * Cf::TILE, &tmX, br, cb * CT_CH, sb * CT_TOK - (W - 1), b);
  };
  if (tid == 0) {
    for (int i = 0; i < CT_STAGES; ++i) mbar_init(&bar[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  pdl_wait();  // the previous kernel's output (this conv's input) is complete
  pdl_trigger();
  if (tid == 0)
    for (int k = 0; k < CT_STAGES; ++k) issue(k);
  {
    // the block's taps and bias through shared memory: thread i reads channel i's W taps (a warp
    // reads one contiguous span) and stores them tap-major; per-thread reads of eight channels'
    // taps straight from global memory touched 32 cache lines per warp load and dominated the kernel
    const int ci = cb * CT_CH + tid;
#pragma unroll
    for (int j = 0; j < W; ++j) wsm[j * CT_CH + tid] = ci < channels ? w[(int64_t)ci * W + j] : 0.f;
    bsm[tid] = (ci < channels && bias) ? bias[ci] : 0.f;
  }
  __syncthreads();
  float wt[8][W], bi[8];
#pragma unroll
  for (int j = 0; j < W; ++j) {
    const float4 a = *reinterpret_cast<const float4*>(wsm + j * CT_CH + tx * 8);
    const float4 c = *reinterpret_cast<const float4*>(wsm + j * CT_CH + tx * 8 + 4);
    wt[0][j] = a.x; wt[1][j] = a.y; wt[2][j] = a.z; wt[3][j] = a.w;
    wt[4][j] = c.x; wt[5][j] = c.y; wt[6][j] = c.z; wt[7][j] = c.w;
  }
  {
    const float4 a = *reinterpret_cast<const float4*>(bsm + tx * 8);
    const float4 c = *reinterpret_cast<const float4*>(bsm + tx * 8 + 4);
    bi[0] = a.x; bi[1] = a.y; bi[2] = a.z; bi[3] = a.w;
    bi[4] = c.x; bi[5] = c.y; bi[6] = c.z; bi[7] = c.w;
  }
  bool ok = true;
  for (int k = 0;; ++k) {
    const int tile = blockIdx.x + k * gridDim.x;
    if (tile >= ntiles) break;
    ok = ok && mbar_wait(&bar[k % CT_STAGES], (k / CT_STAGES) & 1, abort_flag);
    if (ok) {
      // rows past the sequence end and channels past the last read as zero; the store clips them
      const uint8_t* st = sm + (k % CT_STAGES) * Cf::TILE;
      uint8_t* ob = outs + (k & 1) * Cf::OUT;
      const int r0 = ty * 4;
      float in[4 + W - 1][8];
#pragma unroll
      for (int r = 0; r < 4 + W - 1; ++r)
        load8<T>(reinterpret_cast<const T*>(st + (size_t)(r0 + r) * (CT_CH * 2) + tx * 16), in[r]);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float acc = bi[e];
#pragma unroll
          for (int j = 0; j < W; ++j) acc = fmaf(wt[e][j], in[kk + j][e], acc);
          o[e] = act == TH_ACT_SILU ? silu_tanh(acc) : acc;
        }
        store8<T>(reinterpret_cast<T*>(ob + (size_t)(r0 + kk) * (CT_CH * 2) + tx * 16), o);
      }
    }
    fence_proxy_async();  // the output tile (generic writes) -> visible to the TMA store
    // the store of the previous tile has read its buffer, which the next tile writes
    if (tid == 0) bulk_wait_read0();
    __syncthreads();  // everyone is done with this input stage and this output tile
    if (tid == 0 && ok) {
      int sb, b;
      coords(tile, sb, b);
      tma_store_3d(&tmY, outs + (k & 1) * Cf::OUT, cb * CT_CH, sb * CT_TOK, b);
      bulk_commit();
      issue(k + CT_STAGES);
    }
  }
  if (tid == 0) bulk_wait0();  // the output stores are complete before the block exits
}

// ------------------------------------------------------------ embedding
template <typename T>
__global__ void __launch_bounds__(256) embedding_kernel(const int64_t* __restrict__ ids, const T* __restrict__ table,
                                                        int64_t ldt, T* __restrict__ out, int64_t ldo, int64_t tokens,
                                                        int dim, int64_t vocab) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int64_t nw = (int64_t)gridDim.x * 8;
  for (int64_t t = wid; t < tokens; t += nw) {
    int64_t id = ids[t];
    if (id < 0 || id >= vocab) {
      if (lane == 0) atomicOr(&g_device_error, TH_DEVERR_BAD_ARG);
      id = 0;
    }
    const T* src = table + id * ldt;
    T* dst = out + t * ldo;
    for (int c = lane * 8; c < dim; c += 256) *reinterpret_cast<uint4*>(dst + c) = *reinterpret_cast<const uint4*>(src + c);
  }
}

// Blocks of 8 warps for `rows` rows at `per_warp` rows per warp (one pass,
// at most 8 blocks per SM; larger inputs loop).
static unsigned rows_grid(int64_t rows, int per_warp) {
  const int64_t want = (rows + 8 * per_warp - 1) / (8 * per_warp), cap = (int64_t)sm_count() * 8;
  return (unsigned)(want < cap ? (want > 0 ? want : 1) : cap);
}

static unsigned row_grid(int64_t rows) {
  const int64_t per_block = 8;  // warps per 256-thread block
  int64_t want = (rows + per_block - 1) / per_block;
  const int64_t cap = (int64_t)sm_count() * 16;
  return (unsigned)(want < cap ? (want > 0 ? want : 1) : cap);
}

}  // namespace th

extern "C" int th_rowstat(const th_rowstat_args* a, void* stream) {
  using namespace th;
  if (!a || !a->x || !a->sumsq) return fail(TH_EINVAL, "th_rowstat: NULL argument");
  if (a->rows <= 0 || a->cols <= 0 || a->ldx < a->cols || a->cols > INT32_MAX) return fail(TH_EINVAL, "th_rowstat: bad shape");
  if ((a->cols % 8 == 0) && (!aligned16(a->x) || a->ldx % 8)) return fail(TH_EALIGN, "th_rowstat: x must be 16-B aligned with ldx %% 8 == 0");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool small = a->cols <= 1024;
  if (a->dtype != TH_F32 && a->cols % 8 == 0 && a->cols <= 4096) {  // rows in registers, two at a time when short
    const unsigned g = small ? rows_grid(a->rows, 2) : rows_grid(a->rows, 1);
    if (a->dtype == TH_BF16) {
      auto k = small ? rowstat_rows<__nv_bfloat16, 4, 2> : rowstat_rows<__nv_bfloat16, 16, 1>;
      launch_pdl(k, dim3(g), dim3(256), 0, st, (const __nv_bfloat16*)a->x, a->ldx, a->sumsq, a->rows, (int)a->cols);
    } else {
      auto k = small ? rowstat_rows<__half, 4, 2> : rowstat_rows<__half, 16, 1>;
      launch_pdl(k, dim3(g), dim3(256), 0, st, (const __half*)a->x, a->ldx, a->sumsq, a->rows, (int)a->cols);
    }
    return check_launch("th_rowstat");
  }
  const unsigned g = row_grid(a->rows);
  switch (a->dtype) {
    case TH_F32: (small ? rowstat_kernel<float, 4> : rowstat_kernel<float, 16>)<<<g, 256, 0, st>>>((const float*)a->x, a->ldx, a->sumsq, a->rows, (int)a->cols); break;
    case TH_BF16: (small ? rowstat_kernel<__nv_bfloat16, 4> : rowstat_kernel<__nv_bfloat16, 16>)<<<g, 256, 0, st>>>((const __nv_bfloat16*)a->x, a->ldx, a->sumsq, a->rows, (int)a->cols); break;
    case TH_F16: (small ? rowstat_kernel<__half, 4> : rowstat_kernel<__half, 16>)<<<g, 256, 0, st>>>((const __half*)a->x, a->ldx, a->sumsq, a->rows, (int)a->cols); break;
    default: return fail(TH_EDTYPE, "th_rowstat: bad dtype %d", a->dtype);
  }
  return check_launch("th_rowstat");
}

extern "C" int th_rmsnorm(const th_rmsnorm_args* a, void* stream) {
  using namespace th;
  if (!a || !a->x || !a->y) return fail(TH_EINVAL, "th_rmsnorm: NULL argument");
  if (a->rows <= 0 || a->cols <= 0 || a->ldx < a->cols || a->ldy < a->cols || a->cols > INT32_MAX) return fail(TH_EINVAL, "th_rmsnorm: bad shape");
  if ((a->cols % 8 == 0) && (!aligned16(a->x) || !aligned16(a->y) || a->ldx % 8 || a->ldy % 8))
    return fail(TH_EALIGN, "th_rmsnorm: x/y must be 16-B aligned with ld %% 8 == 0");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool small = a->cols <= 1024;
  if (a->dtype != TH_F32 && a->cols % 8 == 0 && a->cols <= 4096) {  // rows in registers, gain in shared memory
    const unsigned g = small ? rows_grid(a->rows, 2) : rows_grid(a->rows, 1);
    const size_t sm = (size_t)a->cols * 4;
    if (a->dtype == TH_BF16) {
      auto k = small ? rmsnorm_rows<__nv_bfloat16, 4, 2> : rmsnorm_rows<__nv_bfloat16, 16, 1>;
      launch_pdl(k, dim3(g), dim3(256), sm, st, (const __nv_bfloat16*)a->x, a->ldx, a->gain, (__nv_bfloat16*)a->y,
                 a->ldy, a->rows, (int)a->cols, a->eps);
    } else {
      auto k = small ? rmsnorm_rows<__half, 4, 2> : rmsnorm_rows<__half, 16, 1>;
      launch_pdl(k, dim3(g), dim3(256), sm, st, (const __half*)a->x, a->ldx, a->gain, (__half*)a->y, a->ldy, a->rows,
                 (int)a->cols, a->eps);
    }
    return check_launch("th_rmsnorm");
  }
  const unsigned g = row_grid(a->rows);
  switch (a->dtype) {
    case TH_F32: (small ? rmsnorm_kernel<float, 4> : rmsnorm_kernel<float, 16>)<<<g, 256, 0, st>>>((const float*)a->x, a->ldx, a->gain, (float*)a->y, a->ldy, a->rows, (int)a->cols, a->eps); break;
    case TH_BF16: (small ? rmsnorm_kernel<__nv_bfloat16, 4> : rmsnorm_kernel<__nv_bfloat16, 16>)<<<g, 256, 0, st>>>((const __nv_bfloat16*)a->x, a->ldx, a->gain, (__nv_bfloat16*)a->y, a->ldy, a->rows, (int)a->cols, a->eps); break;
    case TH_F16: (small ? rmsnorm_kernel<__half, 4> : rmsnorm_kernel<__half, 16>)<<<g, 256, 0, st>>>((const __half*)a->x, a->ldx, a->gain, (__half*)a->y, a->ldy, a->rows, (int)a->cols, a->eps); break;
    default: return fail(TH_EDTYPE, "th_rmsnorm: bad dtype %d", a->dtype);
  }
  return check_launch("th_rmsnorm");
}

template <typename T, int W>
static void launch_conv(const th_conv1d_args* a, cudaStream_t st) {
  const int64_t T_ = (int64_t)a->batch * a->seq;
  constexpr int tok = th::CONV_TY * th::CONV_TPT;
  dim3 grid((unsigned)((a->channels + 255) / 256), (unsigned)((T_ + tok - 1) / tok));
  th::conv1d_kernel<T, W><<<grid, dim3(32, th::CONV_TY), 0, st>>>((const T*)a->x, a->ldx, a->w, a->bias, (T*)a->y, a->ldy,
                                                        a->batch, a->seq, a->channels, a->act);
}

template <typename T, int W>
static int launch_conv_tma(const th_conv1d_args* a, cudaStream_t st) {
  using Cf = th::CtCfg<W>;
  CUtensorMap tm, ty;
  const uint64_t S = (uint64_t)a->seq;
  int rc = th::make_tmap_3d(&tm, a->x, a->dtype, (uint64_t)a->channels, S, (uint64_t)a->batch, (uint64_t)a->ldx * 2,
                            S * a->ldx * 2, th::CT_CH, Cf::ROWS, false);
  if (!rc)
    rc = th::make_tmap_3d(&ty, a->y, a->dtype, (uint64_t)a->channels, S, (uint64_t)a->batch, (uint64_t)a->ldy * 2,
                          S * a->ldy * 2, th::CT_CH, th::CT_TOK, false);
  if (rc) return rc;
  if ((rc = th::smem_limit(th::conv1d_tma<T, W>, Cf::SMEM, "th_conv1d(tma)"))) return rc;
  const int ncb = (a->channels + th::CT_CH - 1) / th::CT_CH, nsb = (a->seq + th::CT_TOK - 1) / th::CT_TOK;
  const int ntiles = ncb * nsb * a->batch;
  // a multiple of ncb blocks (each block keeps one channel block and its weights), two per SM
  int grid = (2 * th::sm_count() / ncb) * ncb;
  if (grid < ncb) grid = ncb;
  if (grid > ntiles) grid = ntiles;
  th::launch_pdl(th::conv1d_tma<T, W>, dim3(grid), dim3(256), Cf::SMEM, st, tm, ty, a->w, a->bias, a->channels, a->act,
                 ncb, nsb, ntiles);
  return th::check_launch("th_conv1d(tma)");
}

template <typename T>
static int conv_dispatch(const th_conv1d_args* a, cudaStream_t st) {
  if constexpr (sizeof(T) == 2) {
    switch (a->width) {
      case 2: return launch_conv_tma<T, 2>(a, st);
      case 3: return launch_conv_tma<T, 3>(a, st);
      case 4: return launch_conv_tma<T, 4>(a, st);
      default: break;
    }
  }
  switch (a->width) {
    case 2: launch_conv<T, 2>(a, st); break;
    case 3: launch_conv<T, 3>(a, st); break;
    case 4: launch_conv<T, 4>(a, st); break;
    default: return th::fail(TH_EUNSUPPORTED, "th_conv1d: width %d not built (2..4)", a->width);
  }
  return th::check_launch("th_conv1d");
}

extern "C" int th_conv1d(const th_conv1d_args* a, void* stream) {
  using namespace th;
  if (!a || !a->x || !a->w || !a->y) return fail(TH_EINVAL, "th_conv1d: NULL argument");
  if (a->batch <= 0 || a->seq <= 0 || a->channels <= 0) return fail(TH_EINVAL, "th_conv1d: bad shape");
  if (a->channels % 8 || a->ldx % 8 || a->ldy % 8 || !aligned16(a->x) || !aligned16(a->y) || a->ldx < a->channels || a->ldy < a->channels)
    return fail(TH_EALIGN, "th_conv1d: channels, ldx, ldy must be multiples of 8 and x/y 16-B aligned");
  if (a->act != TH_ACT_NONE && a->act != TH_ACT_SILU) return fail(TH_EINVAL, "th_conv1d: act must be none or silu");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (a->dtype) {
    case TH_F32: return conv_dispatch<float>(a, st);
    case TH_BF16: return conv_dispatch<__nv_bfloat16>(a, st);
    case TH_F16: return conv_dispatch<__half>(a, st);
    default: return fail(TH_EDTYPE, "th_conv1d: bad dtype %d", a->dtype);
  }
}

extern "C" int th_embedding(const th_embedding_args* a, void* stream) {
  using namespace th;
  if (!a || !a->ids || !a->table || !a->out) return fail(TH_EINVAL, "th_embedding: NULL argument");
  if (a->tokens <= 0 || a->dim <= 0 || a->vocab <= 0) return fail(TH_EINVAL, "th_embedding: bad shape");
  const int eb = elem_bytes(a->dtype);
  if ((a->dim * eb) % 16 || (a->ldt * eb) % 16 || (a->ldo * eb) % 16 || !aligned16(a->table) || !aligned16(a->out))
    return fail(TH_EALIGN, "th_embedding: rows must be 16-B aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned g = row_grid(a->tokens);
  // copy as 8-element vectors of the element type
  switch (a->dtype) {
    case TH_F32:
      // fp32 rows: treat each pair of floats as one 8-byte unit is unnecessary; reuse the 2-byte kernel on a
      // half-typed view with doubled width (a pure byte copy).
      embedding_kernel<__half><<<g, 256, 0, st>>>(a->ids, (const __half*)a->table, a->ldt * 2, (__half*)a->out, a->ldo * 2, a->tokens, (int)(a->dim * 2), a->vocab);
      break;
    case TH_BF16:
    case TH_F16:
      embedding_kernel<__half><<<g, 256, 0, st>>>(a->ids, (const __half*)a->table, a->ldt, (__half*)a->out, a->ldo, a->tokens, (int)a->dim, a->vocab);
      break;
    default: return fail(TH_EDTYPE, "th_embedding: bad dtype %d", a->dtype);
  }
  return check_launch("th_embedding");
}
