// tcgen05 scan pass of the SSD (bf16/fp16 inputs, fp32 accumulation in TMEM).
//
// One CTA per (chunk of 256 rows, head, batch).  With i, j rows of the chunk,
// n the state index and p the head-dim index:
//   phase 1 (tensor cores):  CB  = C . B^T           rows 0-127: j < 128, rows 128-255: j < 256
//                            YO  = C . S_in^T        (S_in: state entering the chunk)
//   phase 2 (CUDA cores):    G   = CB * exp(cumA_i - cumA_j) * dt_j  for j <= i, else 0
//                            written back to shared memory as the bf16 A operand
//   phase 3 (tensor cores):  YD  = G . x
//   phase 4 (CUDA cores):    y = YD + exp(cumA_i) YO + D x_i, gate silu(z), store,
//                            per-head sum of squares (gated RMSNorm statistics)
// TMEM (512 columns): CB rows 0-127 -> cols [0,128), rows 128-255 -> [128,384),
// YO -> [384,448) / [448,512); YD reuses cols [0,64) / [128,192) once CB is read.
// Shared memory: C and B tiles (K-major, 128-byte swizzle, TMA), x (MN-major
// operand of phase 3), S_in (bf16, written by the threads); G reuses the C/B
// space after phase 1.  Below-diagonal 32x32 blocks use
// exp(ci - cj) = exp(ci - c_ref) exp(c_ref - cj) with c_ref the block's last
// column (both factors <= 1), so only diagonal blocks need per-element exps.
#include "common.cuh"

namespace th {

constexpr int TS_L = 256;        // chunk rows
constexpr int TS_P = 64;         // head_dim handled by this path
constexpr uint32_t TS_TMEM = 512;

template <int NS>
struct TsCfg {
  static constexpr int KAT = NS / 64;                 // 64-wide K atoms of the state dim
  static constexpr int C_BYTES = KAT * TS_L * 128;    // [256 rows] x NS, one 32 KB region per atom
  static constexpr int B_BYTES = KAT * TS_L * 128;
  static constexpr int X_BYTES = TS_L * 128;          // [256 rows] x 64
  static constexpr int S_BYTES = KAT * TS_P * 128;    // [64 rows] x NS
  static constexpr int OFF_C = 0, OFF_B = C_BYTES, OFF_X = OFF_B + B_BYTES, OFF_S = OFF_X + X_BYTES;
  // G tiles (phase 2): rows 0-127 ([128 x 128], 32 KB) reuse the C region; rows
  // 128-255 ([128 x 256], 64 KB) reuse the B region when it is that large,
  // otherwise get their own region after S_in.
  static constexpr int G1_BYTES = 4 * 128 * 128;
  static constexpr bool G1_IN_B = B_BYTES >= G1_BYTES;
  static constexpr int OFF_G0 = OFF_C;
  static constexpr int OFF_G1 = G1_IN_B ? OFF_B : OFF_S + S_BYTES;
  static constexpr int OFF_F = (G1_IN_B ? OFF_S + S_BYTES : OFF_G1 + G1_BYTES);  // fp32 scalars
  static constexpr int SMEM = 1024 + OFF_F + 4 * TS_L * 4 + 256;
  static_assert(2 * 128 * 128 <= C_BYTES, "G0 must fit in the C region");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

// byte offset of element (row, col) of a K-major 128B-swizzled tile made of
// 64-column atoms of `rows` x 128 B
__device__ __forceinline__ uint32_t sw128_off(int row, int col, int rows) {
  const int atom = col >> 6, chunk = (col & 63) >> 3, e = col & 7;
  return (uint32_t)(atom * rows * 128 + row * 128 + ((chunk ^ (row & 7)) << 4) + e * 2);
}

template <typename T, int NS>
__global__ void __launch_bounds__(256, 1)
    ssd_scan_tc(const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmX, th_ssd_args p, int nchunks, const float* __restrict__ states,
                const float* __restrict__ cum) {
  using C = TsCfg<NS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_align<1024>(smem_raw);
  float* cs = reinterpret_cast<float*>(sm + C::OFF_F);  // cumA [256]
  float* dts = cs + TS_L;                                // dt [256]
  float* colf = dts + TS_L;                              // exp(c_ref(j) - c_j) dt_j [256]
  float* ecs = colf + TS_L;                              // exp(cumA_i) [256]
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(ecs + TS_L);
  uint64_t* bar_m1 = bar_tma + 1;
  uint64_t* bar_m2 = bar_tma + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar_tma + 3);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hg = h / (p.heads / p.ngroups);
  const int s0 = c * TS_L, len = min(TS_L, p.seq - s0);
  const int64_t t0 = (int64_t)b * p.seq + s0;

  if (tid == 0) {
    mbar_init(bar_tma, 1);
    mbar_init(bar_m1, 1);
    mbar_init(bar_m2, 1);
    *abort_flag = 0;
    fence_mbar_init();
    // TMA: C and B (KAT atoms each), x (one atom)
    constexpr uint32_t bytes = C::C_BYTES + C::B_BYTES + C::X_BYTES;
    mbar_arrive_expect_tx(bar_tma, bytes);
    for (int a = 0; a < C::KAT; ++a) {
      tma_load_2d(sm + C::OFF_C + a * TS_L * 128, &tmC, bar_tma, hg * NS + a * 64, (int)t0);
      tma_load_2d(sm + C::OFF_B + a * TS_L * 128, &tmB, bar_tma, hg * NS + a * 64, (int)t0);
    }
    tma_load_2d(sm + C::OFF_X, &tmX, bar_tma, h * TS_P, (int)t0);
  }
  __syncwarp();
  if (warp == 0) tmem_alloc(tslot, TS_TMEM);
  // scalars: cumA, dt of the chunk (rows >= len are masked below)
  {
    // the state pass wrote cumA for every row of the chunk (padded rows repeat
    // the last value), so every exp below has a non-positive argument
    const float* cp = cum + (((int64_t)b * p.heads + h) * nchunks + c) * TS_L;
    cs[tid] = cp[tid];
    dts[tid] = tid < len ? p.dt[(t0 + tid) * p.lddt + h] : 0.f;
  }
  // S_in (fp32 [64][NS]) -> bf16 K-major swizzled tile
  {
    const float* Sin = states + (((int64_t)b * nchunks + c) * p.heads + h) * (int64_t)(TS_P * NS);
    for (int v = tid; v < TS_P * NS / 8; v += 256) {
      const int r = v / (NS / 8), col = (v % (NS / 8)) * 8;
      float f[8];
      load8<float>(Sin + (int64_t)r * NS + col, f);
      store8<T>(reinterpret_cast<T*>(sm + C::OFF_S + sw128_off(r, col, TS_P)), f);
    }
  }
  __syncthreads();
  {
    const float ci = cs[tid];
    ecs[tid] = __expf(ci);
    const int ref = (tid | 31);  // last column of this 32-column block
    colf[tid] = (tid < len) ? __expf(cs[min(ref, TS_L - 1)] - ci) * dts[tid] : 0.f;
  }
  fence_proxy_async();  // S_in tile written by threads -> visible to the tensor cores
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  // ---------------------------------------------------------------- phase 1
  if (tid == 0) {
    if (mbar_wait(bar_tma, 0, abort_flag)) {
      tc_fence_after();
      const uint32_t cA = smem_u32(sm + C::OFF_C), bA = smem_u32(sm + C::OFF_B), sA = smem_u32(sm + C::OFF_S);
      constexpr int fmt = DT<T>::id == TH_BF16 ? 1 : 0;
      constexpr uint32_t id_cb0 = make_idesc_f16(128, 128, fmt, 0, 0);
      constexpr uint32_t id_cb1 = make_idesc_f16(128, 256, fmt, 0, 0);
      constexpr uint32_t id_yo = make_idesc_f16(128, 64, fmt, 0, 0);
      for (int k = 0; k < NS / 16; ++k) {
        const uint32_t ko = (uint32_t)((k >> 2) * TS_L * 128 + (k & 3) * 32);    // C/B: 256-row atoms
        const uint32_t so = (uint32_t)((k >> 2) * TS_P * 128 + (k & 3) * 32);    // S: 64-row atoms
        const uint64_t a0 = make_desc_sw128(cA + ko, 16, 1024);                 // C rows 0-127
        const uint64_t a1 = make_desc_sw128(cA + ko + 128 * 128, 16, 1024);     // C rows 128-255
        const uint64_t bb = make_desc_sw128(bA + ko, 16, 1024);                 // B rows 0-255
        const uint64_t ss = make_desc_sw128(sA + so, 16, 1024);                 // S_in rows (p) 0-63
        const uint32_t acc = k ? 1u : 0u;
        tc_mma_f16(tmem + 0, a0, bb, id_cb0, acc);
        tc_mma_f16(tmem + 128, a1, bb, id_cb1, acc);
        tc_mma_f16(tmem + 384, a0, ss, id_yo, acc);
        tc_mma_f16(tmem + 448, a1, ss, id_yo, acc);
      }
    }
    tc_commit(bar_m1);
  }
  __syncwarp();
  bool ok1 = mbar_wait(bar_m1, 0, abort_flag);
  ok1 = mbar_wait(bar_tma, 0, abort_flag) && ok1;  // x tile (TMA-written) is read in phase 4
  ok1 = __all_sync(0xffffffffu, ok1);
  __syncwarp();
  tc_fence_after();
  // ---------------------------------------------------------------- phase 2
  // quarter q = warp & 3 owns TMEM lanes 32q..32q+31 (rows r = 32q + lane of
  // either 128-row half).  Warp q:   half 0 cols [0,128) + half 1 cols [0,64)
  //                                warp q+4: half 1 cols [64,256)
  const int q = warp & 3, rloc = q * 32 + lane;
  if (ok1 && !*abort_flag) {
    const uint32_t lanebase = tmem + ((uint32_t)(q * 32) << 16);
    auto do_block = [&](int half, int j0) {
      const int i = half * 128 + rloc;  // chunk row
      float v[32];
      tmem_ld32(lanebase + (half ? 128 : 0) + j0, v);
      const float ci = cs[i];
      if (j0 + 31 <= i) {  // fully below the diagonal: factorised decay
        const float rf = __expf(ci - cs[j0 + 31]);
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] *= rf * colf[j0 + e];
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int j = j0 + e;
          v[e] = (j <= i && j < len) ? v[e] * __expf(ci - cs[j]) * dts[j] : 0.f;
        }
      }
      // write bf16 G into the A-operand tile of this half (K-major, 128B swizzle)
      uint8_t* gbase = sm + (half ? C::OFF_G1 : C::OFF_G0);
#pragma unroll
      for (int e8 = 0; e8 < 32; e8 += 8) store8<T>(reinterpret_cast<T*>(gbase + sw128_off(rloc, j0 + e8, 128)), v + e8);
    };
    if (warp < 4) {
      for (int j0 = 0; j0 < 128; j0 += 32) do_block(0, j0);
      for (int j0 = 0; j0 < 64; j0 += 32) do_block(1, j0);
    } else {
      for (int j0 = 64; j0 < 256; j0 += 32) do_block(1, j0);
    }
  }
  fence_proxy_async();  // G written by threads -> visible to the tensor cores
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // ---------------------------------------------------------------- phase 3
  if (tid == 0) {
    if (ok1 && !*abort_flag) {
      const uint32_t g0 = smem_u32(sm + C::OFF_G0), g1 = smem_u32(sm + C::OFF_G1), xA = smem_u32(sm + C::OFF_X);
      constexpr int fmt = DT<T>::id == TH_BF16 ? 1 : 0;
      constexpr uint32_t id_y = make_idesc_f16(128, 64, fmt, 0, 1);  // B (x) is MN-major
      // half 0: K = j in [0,128)  (2 atoms of 128 rows x 128 B)
      for (int k = 0; k < 8; ++k) {
        const uint64_t ga = make_desc_sw128(g0 + (k >> 2) * 128 * 128 + (k & 3) * 32, 16, 1024);
        const uint64_t xb = make_desc_sw128(xA + k * 16 * 128, TS_L * 128, 1024);
        tc_mma_f16(tmem + 0, ga, xb, id_y, k ? 1u : 0u);
      }
      // half 1: K = j in [0,256)  (4 atoms)
      for (int k = 0; k < 16; ++k) {
        const uint64_t ga = make_desc_sw128(g1 + (k >> 2) * 128 * 128 + (k & 3) * 32, 16, 1024);
        const uint64_t xb = make_desc_sw128(xA + k * 16 * 128, TS_L * 128, 1024);
        tc_mma_f16(tmem + 128, ga, xb, id_y, k ? 1u : 0u);
      }
    }
    tc_commit(bar_m2);
  }
  __syncwarp();
  const bool ok2 = __all_sync(0xffffffffu, mbar_wait(bar_m2, 0, abort_flag) && ok1 && !*abort_flag);
  __syncwarp();
  tc_fence_after();
  // ---------------------------------------------------------------- phase 4
  if (ok2) {
    const int half = warp >> 2;
    const int i = half * 128 + rloc;
    const uint32_t lanebase = tmem + ((uint32_t)(q * 32) << 16);
    float yd[64], yo[64];
    tmem_ld32(lanebase + (half ? 128 : 0), yd);
    tmem_ld32(lanebase + (half ? 128 : 0) + 32, yd + 32);
    tmem_ld32(lanebase + (half ? 448 : 384), yo);
    tmem_ld32(lanebase + (half ? 448 : 384) + 32, yo + 32);
    if (i < len) {
      const int64_t t = t0 + i;
      const float e_i = ecs[i];
      const float Dh = p.D ? p.D[h] : 0.f;
      const T* zrow = p.z ? reinterpret_cast<const T*>(p.z) + t * p.ldz + (int64_t)h * TS_P : nullptr;
      T* orow = reinterpret_cast<T*>(p.out) + t * p.ldo + (int64_t)h * TS_P;
      float ss = 0.f;
#pragma unroll
      for (int c8 = 0; c8 < TS_P; c8 += 8) {
        float xv[8], zv[8], o[8];
        load8<T>(reinterpret_cast<const T*>(sm + C::OFF_X + sw128_off(i, c8, TS_L)), xv);
        if (zrow) load8<T>(zrow + c8, zv);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float y = yd[c8 + e] + e_i * yo[c8 + e] + Dh * xv[e];
          if (zrow) y *= silu_f(zv[e]);
          o[e] = y;
        }
        store8<T>(orow + c8, o);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float qv = round_to<T>(o[e]);
          ss += qv * qv;
        }
      }
      if (p.gss) p.gss[t * p.ldgss + h] = ss;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, TS_TMEM);
}

// Applies to 2-byte dtypes, head_dim 64, state_dim 64 or 128, chunk 256 and
// 16-byte aligned rows; returns 1 (not taken) otherwise.
template <typename T>
static int ssd_scan_tc_try(const th_ssd_args* a, int nchunks, const float* states, const float* cum, cudaStream_t st,
                           int* rc) {
  if (a->head_dim != TS_P || a->chunk != TS_L || (a->state_dim != 64 && a->state_dim != 128)) return 1;
  if (!aligned16(a->x) || !aligned16(a->B) || !aligned16(a->C) || !aligned16(a->out) || a->ldx % 8 || a->ldb % 8 ||
      a->ldc % 8 || a->ldo % 8)
    return 1;
  if (a->z && (!aligned16(a->z) || a->ldz % 8)) return 1;
  const int64_t T_ = (int64_t)a->batch * a->seq;
  const uint64_t gn = (uint64_t)a->ngroups * a->state_dim;
  CUtensorMap tc_, tb_, tx_;
  int r = make_tmap_2d(&tc_, a->C, a->dtype, gn, (uint64_t)T_, (uint64_t)a->ldc * 2, 64, TS_L, true);
  if (!r) r = make_tmap_2d(&tb_, a->B, a->dtype, gn, (uint64_t)T_, (uint64_t)a->ldb * 2, 64, TS_L, true);
  if (!r) r = make_tmap_2d(&tx_, a->x, a->dtype, (uint64_t)a->heads * TS_P, (uint64_t)T_, (uint64_t)a->ldx * 2, 64, TS_L, true);
  if (r) { *rc = r; return 0; }
  dim3 grid((unsigned)nchunks, (unsigned)a->heads, (unsigned)a->batch);
  if (a->state_dim == 128) {
    using Cf = TsCfg<128>;
    if ((*rc = smem_limit(ssd_scan_tc<T, 128>, Cf::SMEM, "th_ssd(scan, tcgen05)"))) return 0;
    ssd_scan_tc<T, 128><<<grid, 256, Cf::SMEM, st>>>(tc_, tb_, tx_, *a, nchunks, states, cum);
  } else {
    using Cf = TsCfg<64>;
    if ((*rc = smem_limit(ssd_scan_tc<T, 64>, Cf::SMEM, "th_ssd(scan, tcgen05)"))) return 0;
    ssd_scan_tc<T, 64><<<grid, 256, Cf::SMEM, st>>>(tc_, tb_, tx_, *a, nchunks, states, cum);
  }
  *rc = check_launch("th_ssd(scan, tcgen05)");
  return 0;
}

}  // namespace th
