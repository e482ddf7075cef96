// Chunked SSD on tcgen05 in two launches (2-byte dtypes, head_dim 64,
// chunk 256, state_dim 128).  With l, i, j rows of a chunk, n the state
// index and p the head-dim index:
//
// ssd_state_tc -- one CTA per (head, batch) walks the chunks in order and
//   keeps the running state S[n][p] (fp32) in TMEM:
//     cum_l = sum_{l' <= l} dt_l' A            (inclusive, per chunk)
//     w_l   = exp(cum_last - cum_l) dt_l       (<= dt_l)
//     S    <- exp(cum_last) S + B^T (w . x)     (one M=128 N=64 K=256 MMA per chunk,
//                                               B^T and x MN-major straight from TMA)
//   Before a chunk's update it stores the state entering that chunk (bf16
//   [n][p], the scan's operand) and writes the chunk's scalars for the scan:
//   cum, dt and colf_l = exp(cum_{l|31} - cum_l) dt_l.  This replaces the
//   separate chunk-state and inter-chunk passes and their fp32 round trips.
//
// ssd_scan_g -- one CTA per (chunk, set of heads, batch), in two passes:
//   query rows 128-255 (256 keys), then rows 0-127 (128 keys), so every CTA
//   carries the same work.  The heads of one B/C group share C.B^T, so each
//   pass computes it once into TMEM and then, head by head:
//     G = C.B^T * exp(cum_i - cum_j) dt_j  (j <= i), plus D on the diagonal
//         (CUDA cores, TMEM -> packed fp32 pairs -> bf16 back into TMEM)
//     Y = G . x + exp(cum_i) (C . S_in)     (tcgen05, G the A operand from TMEM)
//     y = Y * silu(z) -> shared memory -> TMA store, per-head sum of y^2
//   D on the diagonal of G makes G . x carry the D x skip.  Sub-diagonal
//   blocks use exp(ci - cj) = exp(ci - c_ref) exp(c_ref - cj) with c_ref the
//   32-key block's last column (neither factor overflows).
//
// Every wait is bounded; on a timeout the roles skip their work but still
// pass every barrier, so the CTA always drains and frees TMEM.
#include "common.cuh"

namespace th {

constexpr int CK_L = 256, CK_P = 64, CK_NS = 128;
// Per (batch, head, chunk) scalar record written by the state kernel:
// cum[256] | dt[256] | colf[256] | D, 0, 0, 0   (fp32, 3088 bytes)
constexpr int CK_SCAL = 3 * CK_L + 4;
constexpr int CK_SR = 4;  // scalar ring depth of the scan

inline size_t ck_scal_bytes(int batch, int heads, int nc) {
  return ((size_t)batch * heads * nc * CK_SCAL * 4 + 1023) & ~size_t(1023);
}
// scalar records | S_in (bf16, one slot per chunk; slot 0 unused) | S_c (bf16; last slot unused)
inline size_t ck_state_bytes(int batch, int nc, int heads, int ns, int p) {
  return (size_t)batch * nc * heads * ns * p * 2;
}
inline size_t ck_ws_bytes(int batch, int seq, int heads, int ns, int p = CK_P) {
  const int nc = (seq + CK_L - 1) / CK_L;
  return ck_scal_bytes(batch, heads, nc) + 2 * ck_state_bytes(batch, nc, heads, ns, p);
}

__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// ------------------------------------------------------------------ states
struct StC {
  static constexpr int B_BYTES = 2 * CK_L * 128;  // two 64-wide state atoms x 256 rows
  static constexpr int X_BYTES = CK_L * 128;
  static constexpr int DT_BYTES = CK_L * 16;      // dt of 4 heads x 256 rows (fp32)
  static constexpr int STAGE = B_BYTES + X_BYTES + DT_BYTES;
  static constexpr int OFF_SIN = 2 * STAGE;          // state staging [128 n][64 p]
  static constexpr int OFF_REC = OFF_SIN + 128 * 128;  // scalar record staging
  static constexpr int OFF_F = OFF_REC + CK_SCAL * 4;  // cum[256], w[256], warp totals[8]
  static constexpr int OFF_BAR = OFF_F + (2 * CK_L + 8) * 4;
  static constexpr int SMEM = 1024 + OFF_BAR + 64;
  static_assert(OFF_SIN % 1024 == 0 && OFF_REC % 16 == 0, "alignment");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

constexpr int ST_PF = 3;  // chunks of L2 prefetch ahead of the two stages

template <typename T>
__global__ void __launch_bounds__(320, 1)
    ssd_state_tc(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmX,
                 const __grid_constant__ CUtensorMap tmDT, const __grid_constant__ CUtensorMap tmS, th_ssd_args p,
                 int nc, float* __restrict__ scal) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_align<1024>(smem_raw);
  float* rec = reinterpret_cast<float*>(sm + StC::OFF_REC);
  float* cums = reinterpret_cast<float*>(sm + StC::OFF_F);
  float* wsm = cums + CK_L;
  float* wtot = wsm + CK_L;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + StC::OFF_BAR);
  uint64_t* empty = full + 2;
  uint64_t* ready = full + 4;
  uint64_t* done = full + 5;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(full + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = h / (p.heads / p.ngroups);

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
    mbar_init(ready, 256);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tslot, 128);  // two chunk-state buffers
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  pdl_wait();  // the previous kernel's outputs (this kernel's inputs) are complete
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // L2 prefetch of the chunks ahead of the two smem stages (each chunk's loads are ~100 KB and the
      // walk is serial: without it the loads' latency sets the pace)
      auto prefetch = [&](int c) {
        tma_prefetch_3d(&tmB, g * CK_NS, c * CK_L, b);
        tma_prefetch_3d(&tmB, g * CK_NS + 64, c * CK_L, b);
        tma_prefetch_3d(&tmX, h * CK_P, c * CK_L, b);
        tma_prefetch_3d(&tmDT, h & ~3, c * CK_L, b);
      };
      for (int c = 2; c < min(2 + ST_PF, nc); ++c) prefetch(c);
      for (int c = 0; c < nc; ++c) {
        const int s = c & 1;
        if (c + 2 + ST_PF < nc) prefetch(c + 2 + ST_PF);
        if (c >= 2 && !mbar_wait(&empty[s], ((c >> 1) - 1) & 1, abort_flag)) break;
        uint8_t* st = sm + s * StC::STAGE;
        mbar_arrive_expect_tx(&full[s], StC::STAGE);
        tma_load_3d(st, &tmB, &full[s], g * CK_NS, c * CK_L, b);
        tma_load_3d(st + CK_L * 128, &tmB, &full[s], g * CK_NS + 64, c * CK_L, b);
        tma_load_3d(st + StC::B_BYTES, &tmX, &full[s], h * CK_P, c * CK_L, b);
        tma_load_3d(st + StC::B_BYTES + StC::X_BYTES, &tmDT, &full[s], h & ~3, c * CK_L, b);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr int fmt = DT<T>::id == TH_BF16 ? 1 : 0;
      constexpr uint32_t idesc = make_idesc_f16(128, 64, fmt, 1, 1);  // A = B^T and B = x, both MN-major
      for (int c = 0; c < nc; ++c) {
        if (!mbar_wait(ready, c & 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t st = smem_u32(sm + (c & 1) * StC::STAGE);
        for (int k = 0; k < CK_L / 16; ++k) {
          const uint64_t ad = make_desc_sw128(st + k * 2048, CK_L * 128, 1024);
          const uint64_t bd = make_desc_sw128(st + StC::B_BYTES + k * 2048, CK_L * 128, 1024);
          tc_mma_f16(tmem + (c & 1) * 64, ad, bd, idesc, k > 0 ? 1u : 0u);  // the chunk's own state, fresh
        }
        tc_commit(done);
        tc_commit(&empty[c & 1]);
      }
    }
  } else {
    // 256 math threads: token / x row l = mt; TMEM quadrant q, state columns half*32..+32
    const int mt = tid - 64;
    const int wm = warp - 2;  // math warp 0..7
    const int q = warp & 3, half = wm >> 2;
    const int n = q * 32 + lane;
    const float Ah = p.A[h];
    const float Dh = p.D ? p.D[h] : 0.f;
    bool ok = true;
    float srun[32];  // running state S_in, rows n, columns half*32.. (fp32)
#pragma unroll
    for (int e = 0; e < 32; ++e) srun[e] = 0.f;
    float prev_total = 0.f;
    for (int c = 0; c < nc; ++c) {
      uint8_t* st = sm + (c & 1) * StC::STAGE;
      ok = ok && mbar_wait(&full[c & 1], (c >> 1) & 1, abort_flag);
      // inclusive prefix sum of dt*A over the chunk (rows past the sequence were zero-filled by TMA)
      const int l = mt;
      const float* dtv = reinterpret_cast<const float*>(st + StC::B_BYTES + StC::X_BYTES);
      const float d = ok ? dtv[l * 4 + (h & 3)] : 0.f;
      float v = d * Ah;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      if (lane == 31) wtot[wm] = v;
      if (mt == 0) bulk_wait_read0();  // the previous chunk's stores have read their staging
      named_bar(1, 256);
      float off = 0.f, total = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const float t = wtot[w];
        off += w < wm ? t : 0.f;
        total += t;
      }
      const float cl = off + v;
      cums[l] = cl;
      const float w_l = __expf(total - cl) * d;
      named_bar(1, 256);
      // the chunk's scalar record for the scan
      rec[l] = cl;
      rec[CK_L + l] = d;
      rec[2 * CK_L + l] = __expf(cums[l | 31] - cl) * d;
      if (mt == 0) *reinterpret_cast<float4*>(rec + 3 * CK_L) = make_float4(Dh, 0.f, 0.f, 0.f);
      // x row l scaled by w_l, in place (whole row: the swizzle only permutes 16-byte chunks)
      if (ok) {
        T* row = reinterpret_cast<T*>(st + StC::B_BYTES + l * 128);
#pragma unroll
        for (int i8 = 0; i8 < 8; ++i8) {  // chunks in swizzled order: no bank conflicts across rows
          const int e8 = (i8 ^ (l & 7)) * 8;
          float f[8];
          load8<T>(row + e8, f);
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] *= w_l;
          store8<T>(row + e8, f);
        }
      }
      fence_proxy_async();  // scaled x (read by the MMA) and the record staging (read by its store)
      tc_fence_before();
      mbar_arrive(ready);   // the MMA of chunk c may start
      // the state entering chunk c (c >= 1): S_in(c) = exp(total(c-1)) S_in(c-1) + S(c-1), with S(c-1)
      // the previous chunk's own state from its MMA; kept in fp32 registers, staged in bf16 for the scan
      if (c > 0) {
        ok = ok && mbar_wait(done, (c - 1) & 1, abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
          tc_fence_after();
          float sv[32];
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + ((c - 1) & 1) * 64 + half * 32, sv);
          tc_fence_before();
          const float f = __expf(prev_total);
          uint8_t* sst = sm + StC::OFF_SIN;
#pragma unroll
          for (int e = 0; e < 32; ++e) srun[e] = fmaf(f, srun[e], sv[e]);
#pragma unroll
          for (int e8 = 0; e8 < 32; e8 += 8)
            store8<T>(reinterpret_cast<T*>(sst + sw128_off(n, half * 32 + e8, 128)), srun + e8);
        }
      }
      fence_proxy_async();  // the state staging (read by its store)
      named_bar(1, 256);
      if (mt == 0 && ok) {
        bulk_store(scal + (((int64_t)b * p.heads + h) * nc + c) * CK_SCAL, rec, CK_SCAL * 4);
        if (c > 0) tma_store_2d(&tmS, sm + StC::OFF_SIN, 0, (((b * nc + c) * p.heads) + h) * CK_NS);
        bulk_commit();
      }
      prev_total = total;
    }
    mbar_wait(done, (nc - 1) & 1, abort_flag);  // the last update finishes before TMEM is freed
    if (mt == 0) bulk_wait0();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 128);
}

// ------------------------------------------------- chunk states, parallel
// ssd_chunk_states -- a persistent kernel over units (batch, chunk, head,
//   128-row half of the state), consecutive units sharing the chunk's B: per
//   unit it computes the chunk's scalars (cum, dt, colf and D, written when
//   the unit is the state's first half), scales x rows by w_l and forms the
//   chunk's own state S_c = B^T (w . x) with one M=128 N=64 K=256 MMA, stored
//   bf16.  Two shared-memory stages and two TMEM buffers overlap the loads of
//   unit j+1, the MMA of unit j and the state store of unit j-1.  The last
//   chunk's state is not needed and is not formed.
// ssd_state_pass -- the inter-chunk recurrence in fp32, elementwise over the
//   state: S_in(c+1) = exp(cum_last(c)) S_in(c) + S_c(c), stored bf16 for
//   the scan.
struct SpC {
  static constexpr int B_BYTES = 2 * CK_L * 128;  // two 64-wide state atoms x 256 rows
  static constexpr int X_BYTES = CK_L * 128;
  static constexpr int DT_BYTES = CK_L * 16;      // dt of 4 heads x 256 rows (fp32)
  static constexpr int STAGE = B_BYTES + X_BYTES + DT_BYTES;
  static constexpr int OFF_F = 2 * STAGE;         // warp totals, two sets of 8
  static constexpr int OFF_BAR = OFF_F + 64;
  static constexpr int SMEM = 1024 + OFF_BAR + 128;
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

template <typename T>
__global__ void __launch_bounds__(320, 1)
    ssd_chunk_states(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmX,
                     const __grid_constant__ CUtensorMap tmDT, th_ssd_args p, int nc, float* __restrict__ scal,
                     T* __restrict__ sc) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_align<1024>(smem_raw);
  float* wtot = reinterpret_cast<float*>(sm + SpC::OFF_F);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + SpC::OFF_BAR);
  uint64_t* empty = full + 2;
  uint64_t* ready = full + 4;
  uint64_t* tdone = full + 6;
  uint64_t* tfree = full + 8;
  uint64_t* fin = full + 10;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(full + 11);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = p.heads, NS = p.state_dim;
  const int nhalf = (NS + 127) / 128;  // 128-row halves of the state (one for d_state 64)
  const int units = p.batch * nc * H * nhalf;
  const int hpg = H / p.ngroups;
  auto need = [&](int u) { return (u / (H * nhalf)) % nc < nc - 1; };  // the chunk's state is used

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
      mbar_init(&ready[i], 256);
      mbar_init(&tdone[i], 1);
      mbar_init(&tfree[i], 8);
    }
    mbar_init(fin, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tslot, 128);  // two unit-state buffers of 64 columns
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  pdl_wait();  // the previous kernel's outputs (this kernel's inputs) are complete
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer
      int j = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x, ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&empty[s], ((j >> 1) - 1) & 1, abort_flag)) break;
        const int nh = u % nhalf, h = (u / nhalf) % H, c = (u / (nhalf * H)) % nc, b = u / (nhalf * H * nc);
        const int g = h / hpg;
        uint8_t* st = sm + s * SpC::STAGE;
        const bool nd = need(u);
        mbar_arrive_expect_tx(&full[s], nd ? (NS >= 128 ? SpC::STAGE : SpC::STAGE - CK_L * 128) : SpC::DT_BYTES);
        if (nd) {
          tma_load_3d(st, &tmB, &full[s], g * NS + nh * 128, c * CK_L, b);
          if (NS >= 128) tma_load_3d(st + CK_L * 128, &tmB, &full[s], g * NS + nh * 128 + 64, c * CK_L, b);
          tma_load_3d(st + SpC::B_BYTES, &tmX, &full[s], h * CK_P, c * CK_L, b);
        }
        tma_load_3d(st + SpC::B_BYTES + SpC::X_BYTES, &tmDT, &full[s], h & ~3, c * CK_L, b);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      constexpr int fmt = DT<T>::id == TH_BF16 ? 1 : 0;
      constexpr uint32_t idesc = make_idesc_f16(128, 64, fmt, 1, 1);  // A = B^T and B = x, both MN-major
      int j = 0, k = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x, ++j) {
        const int s = j & 1;
        if (!mbar_wait(&ready[s], (j >> 1) & 1, abort_flag)) break;
        if (!need(u)) {  // scalars only: hand the stage back
          mbar_arrive(&empty[s]);
          continue;
        }
        if (k >= 2 && !mbar_wait(&tfree[k & 1], ((k >> 1) - 1) & 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t st = smem_u32(sm + s * SpC::STAGE);
        for (int kk = 0; kk < CK_L / 16; ++kk) {
          const uint64_t ad = make_desc_sw128(st + kk * 2048, CK_L * 128, 1024);
          const uint64_t bd = make_desc_sw128(st + SpC::B_BYTES + kk * 2048, CK_L * 128, 1024);
          tc_mma_f16(tmem + (k & 1) * 64, ad, bd, idesc, kk > 0 ? 1u : 0u);
        }
        tc_commit(&tdone[k & 1]);
        tc_commit(&empty[s]);
        ++k;
      }
      tc_commit(fin);  // tracks every MMA this thread issued
    }
  } else {
    // 256 math threads: token row l = mt for the scalars and x; for a state
    // store, row n = q*32 + lane of TMEM quadrant q, columns half*32..+32
    const int mt = tid - 64, wm = warp - 2;
    const int q = warp & 3, half = wm >> 2;
    const int n = q * 32 + lane;
    bool ok = true;
    int j = 0, k = 0;
    int pu = -1;  // the previous unit whose state waits to be stored
    auto store_state = [&](int u, int kb) {  // TMEM buffer kb & 1 -> S_c of unit u
      ok = ok && mbar_wait(&tdone[kb & 1], (kb >> 1) & 1, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        float sv[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (kb & 1) * 64 + half * 32, sv);
        tc_fence_before();
        const int nh = u % nhalf, h = (u / nhalf) % H, c = (u / (nhalf * H)) % nc, b = u / (nhalf * H * nc);
        const int row = nh * 128 + n;
        if (row < NS) {
          T* dst = sc + ((((int64_t)b * nc + c) * H + h) * NS + row) * CK_P + half * 32;
#pragma unroll
          for (int e8 = 0; e8 < 32; e8 += 8) store8<T>(dst + e8, sv + e8);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&tfree[kb & 1]);
    };
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++j) {
      const int s = j & 1;
      const int nh = u % nhalf, h = (u / nhalf) % H, c = (u / (nhalf * H)) % nc, b = u / (nhalf * H * nc);
      const bool nd = need(u);
      uint8_t* st = sm + s * SpC::STAGE;
      ok = ok && mbar_wait(&full[s], (j >> 1) & 1, abort_flag);
      // inclusive prefix sum of dt*A over the chunk (rows past the sequence were zero-filled by TMA)
      const int l = mt;
      const float* dtv = reinterpret_cast<const float*>(st + SpC::B_BYTES + SpC::X_BYTES);
      const float d = ok ? dtv[l * 4 + (h & 3)] : 0.f;
      float v = d * p.A[h];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
      }
      float* wt = wtot + (j & 1) * 8;  // two sets: a warp is at most one unit ahead of the others
      if (lane == 31) wt[wm] = v;
      named_bar(1, 256);
      float off = 0.f, total = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const float t = wt[w];
        off += w < wm ? t : 0.f;
        total += t;
      }
      const float cl = off + v;
      const float c_last31 = __shfl_sync(0xffffffffu, cl, 31);  // cum of row l | 31
      if (nh == 0) {  // the chunk's scalar record for the scan
        float* rec = scal + (((int64_t)b * H + h) * nc + c) * CK_SCAL;
        rec[l] = cl;
        rec[CK_L + l] = d;
        rec[2 * CK_L + l] = __expf(c_last31 - cl) * d;
        if (mt == 0) *reinterpret_cast<float4*>(rec + 3 * CK_L) = make_float4(p.D ? p.D[h] : 0.f, 0.f, 0.f, 0.f);
      }
      if (nd && ok) {  // x row l scaled by w_l = exp(total - cum_l) dt_l, in place, chunks in swizzled order
        const float w_l = __expf(total - cl) * d;
        T* xr = reinterpret_cast<T*>(st + SpC::B_BYTES + l * 128);
#pragma unroll
        for (int i8 = 0; i8 < 8; ++i8) {
          const int e8 = (i8 ^ (l & 7)) * 8;
          float f[8];
          load8<T>(xr + e8, f);
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] *= w_l;
          store8<T>(xr + e8, f);
        }
      }
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(&ready[s]);
      // the previous unit's state leaves while this unit's MMA runs
      if (pu >= 0) {
        store_state(pu, k - 1);
        pu = -1;
      }
      if (nd) {
        pu = u;
        ++k;
      }
    }
    if (pu >= 0) store_state(pu, k - 1);
    if (tid == 64) {  // bounded: the MMAs retire before TMEM is freed, also after an abort
      volatile int dummy = 0;
      mbar_wait(fin, 0, &dummy);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 128);
}

// S_in(0) = 0; S_in(c+1) = exp(cum_last(c)) S_in(c) + S_c(c), four state
// elements per thread, fp32 running state; S_in(c) stored for c >= 1.
template <typename T>
__global__ void __launch_bounds__(256) ssd_state_pass(th_ssd_args p, int nc, const float* __restrict__ scal,
                                                      const T* __restrict__ sc, T* __restrict__ sin) {
  pdl_wait();
  pdl_trigger();
  const int h = blockIdx.y, b = blockIdx.z;
  const int64_t per = (int64_t)p.state_dim * CK_P;  // elements of one state
  const int64_t e = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (e >= per) return;
  float sv[4] = {0.f, 0.f, 0.f, 0.f};
  const float* rec = scal + ((int64_t)b * p.heads + h) * nc * CK_SCAL;
  for (int c = 0; c + 1 < nc; ++c) {
    const int64_t slot = (((int64_t)b * nc + c) * p.heads + h) * per + e;
    const uint2 raw = *reinterpret_cast<const uint2*>(sc + slot);
    const T* hv = reinterpret_cast<const T*>(&raw);
    const float f = __expf(rec[(int64_t)c * CK_SCAL + CK_L - 1]);
#pragma unroll
    for (int i = 0; i < 4; ++i) sv[i] = fmaf(f, sv[i], to_f32(hv[i]));
    uint2 o;
    T* ov = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) ov[i] = from_f32<T>(sv[i]);
    *reinterpret_cast<uint2*>(sin + slot + per * p.heads) = o;  // slot of chunk c + 1
  }
}

// -------------------------------------------------------------------- scan
struct ScMaps {
  CUtensorMap C, B256, B128, X256, X128, S, Y, Z;
};

// ------------------------------------------------------- scan, G in TMEM
// ssd_scan_g -- the scan with the decay-masked operand G held in tensor
// memory and separate warp groups for building G and for the epilogue, so
// head k's epilogue runs while head k+1's G is built and head k+1's MMAs
// run.  One CTA per (chunk, head set, batch; query
// rows 128-255 against 256 keys, then rows 0-127 against 128 keys).
//
// TMEM (512 columns): C.B^T fp32 in [0, 256) (one column per key), a ring of
// two G units in [256, 384) (a unit is 128 keys as 16-bit pairs, 64
// columns; a head is two units in the 256-key pass, one in the 128-key
// pass), and Y (64 columns, G.x) | Yo (64 columns, C.S_in) in [384, 512).
// G is the A operand of the G.x MMA straight from TMEM.
//
// Shared memory: C (128 query rows), B (until C.B^T is in TMEM; then the
// region holds a ring of four z | y tiles), x | S_in stages, the scalar ring
// and the sum-of-squares partials.
//
// Warps: 0 TMA producer (C, B, x | S_in, scalars); 1 MMA issuer; 2-17 build G
// (four per TMEM lane quadrant, each taking two of a unit's eight 16-key
// sub-blocks); 18-25 epilogue (two per quadrant, 32 of the 64 head-dim
// columns each), whose first thread also loads z and stores y by TMA.
template <int NS>
struct SgCfg {
  static constexpr int KAT = NS / 64;                  // 64-wide state atoms
  static constexpr int KB = KAT < 2 ? KAT : 2;         // B atoms resident at a time
  static constexpr int C_BYTES = KAT * 128 * 128;      // 128 query rows
  static constexpr int B_BYTES = KB * CK_L * 128;      // up to 256 keys
  static constexpr int TILE = 128 * 128;               // one z | y tile: 128 rows x 64 columns
  static constexpr int ZS = 4;                         // z | y ring depth
  static constexpr int BZ_BYTES = B_BYTES > ZS * TILE ? B_BYTES : ZS * TILE;
  static constexpr int X_BYTES = CK_L * 128;
  static constexpr int S_BYTES = NS * 128;
  static constexpr int STAGES = NS > 128 ? 1 : 2;
  static constexpr int STAGE = X_BYTES + S_BYTES;
  static constexpr int OFF_C = 0, OFF_B = C_BYTES, OFF_ZY = OFF_B;
  static constexpr int OFF_X = OFF_B + BZ_BYTES;
  static constexpr int OFF_SC = OFF_X + STAGES * STAGE;
  static constexpr int OFF_R = OFF_SC + CK_SR * CK_SCAL * 4;  // [2 heads][2 halves][128] partial sums of y^2
  static constexpr int OFF_BAR = OFF_R + 2 * 2 * 128 * 4;
  static constexpr int SMEM = 1024 + OFF_BAR + 256;
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(OFF_X % 1024 == 0 && OFF_ZY % 1024 == 0, "128-byte swizzle atoms");
};

constexpr int SG_BUILD_WARPS = 16, SG_EPI_WARPS = 8;
constexpr int SG_THREADS = 64 + 32 * (SG_BUILD_WARPS + SG_EPI_WARPS);
constexpr int SG_PF = 4;  // heads of L2 prefetch ahead of the loads
constexpr uint32_t SG_T_G = 256, SG_T_Y = 384;  // TMEM columns of the G ring and of Y | Yo

// The G factors of a 16-key sub-block whose decay span exceeds exp(80) (so the
// factored exp(ci - c_ref) exp(c_ref - cj) could overflow): one exponential
// per element, exp(ci - cj) dt_j <= dt_j for the kept j <= i; the masked
// j > i may overflow and are zeroed by the caller.  Kept out of line so the
// common path keeps its registers.
__device__ __noinline__ void ssd_g_decay_slow(uint32_t (&raw)[16], const float* cum, const float* dts, float ci) {
  for (int e = 0; e < 16; ++e) raw[e] = __float_as_uint(__uint_as_float(raw[e]) * (__expf(ci - cum[e]) * dts[e]));
}

template <typename T, int NS>
__global__ void __maxnreg__(72)
    ssd_scan_g(const __grid_constant__ ScMaps mp, th_ssd_args p, int nc, int hs, int nsets,
               const float* __restrict__ scal) {
  using Cf = SgCfg<NS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_align<1024>(smem_raw);
  float* red = reinterpret_cast<float*>(sm + Cf::OFF_R);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + Cf::OFF_BAR);
  uint64_t* cb_full = bar + 0;
  uint64_t* cb_done = bar + 1;
  uint64_t* b_free = bar + 2;    // d_state 256: the first half of B has been read by the C.B^T MMA
  uint64_t* x_full = bar + 3;    // [2]
  uint64_t* x_empty = bar + 5;   // [2]
  uint64_t* g_full = bar + 7;    // [2] G unit written (by every builder warp)
  uint64_t* g_free = bar + 9;    // [2] G unit read by its MMAs
  uint64_t* y_full = bar + 11;   // Y | Yo of a head complete
  uint64_t* y_empty = bar + 12;  // Y | Yo read by the 8 epilogue warps
  uint64_t* sc_full = bar + 13;  // [CK_SR]
  uint64_t* sc_free = bar + 17;  // [CK_SR] read by every builder and epilogue warp
  uint64_t* z_full = bar + 21;   // [4] z tile landed (or the tile is free, without a gate)
  constexpr int NBAR = 25;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int hpg = p.heads / p.ngroups;
  int u = (int)blockIdx.x;
  const int set = u % (p.ngroups * nsets);
  u /= p.ngroups * nsets;
  const int c = u % nc, b = u / nc;
  const int g = set / nsets, h0 = g * hpg + (set % nsets) * hs;
  const int hcount = min(hs, g * hpg + hpg - h0);
  const int s0 = c * CK_L, len = min(CK_L, p.seq - s0);
  if (hcount <= 0) return;  // nothing to compute (uniform over the CTA)
  const bool has_s = c > 0, has_z = p.z != nullptr;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) *abort_flag = 0;
  if (warp == 1) tmem_alloc(tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  pdl_wait();  // the previous kernel's outputs (this kernel's inputs) are complete
  pdl_trigger();
  for (int pass = 0; pass < 2; ++pass) {
    const int qb = 1 - pass;
    if (qb * 128 >= len) continue;  // a chunk of at most 128 rows has no second half (uniform)
    const int nk = qb ? 256 : 128;
    const int upk = nk / 128;       // G units per head
    if (tid == 0) {  // fresh barriers for each pass (the previous pass has fully drained)
      if (pass > 0)
        for (int i = 0; i < NBAR; ++i) mbar_inval(&bar[i]);
      mbar_init(cb_full, 1);
      mbar_init(cb_done, 1);
      mbar_init(b_free, 1);
      for (int i = 0; i < 2; ++i) {
        mbar_init(&x_full[i], 1);
        mbar_init(&x_empty[i], 1);
        mbar_init(&g_full[i], SG_BUILD_WARPS);
        mbar_init(&g_free[i], 1);
      }
      mbar_init(y_full, 1);
      mbar_init(y_empty, 8);
      for (int i = 0; i < CK_SR; ++i) { mbar_init(&sc_full[i], 1); mbar_init(&sc_free[i], SG_BUILD_WARPS + SG_EPI_WARPS); }
      for (int i = 0; i < 4; ++i) mbar_init(&z_full[i], 1);
      fence_mbar_init();
    }
    __syncthreads();
    const float* scal_bc = scal + ((int64_t)b * p.heads * nc + c) * CK_SCAL;  // + head * nc * CK_SCAL

    if (warp == 0) {
      // ------------------------------------------------ TMA producer
      if (lane == 0) {
        const CUtensorMap* tB = qb ? &mp.B256 : &mp.B128;
        const CUtensorMap* tX = qb ? &mp.X256 : &mp.X128;
        auto load_xs = [&](int k) {
          const int s = Cf::STAGES == 2 ? (k & 1) : 0;
          uint8_t* st = sm + Cf::OFF_X + s * Cf::STAGE;
          mbar_arrive_expect_tx(&x_full[s], nk * 128 + (has_s ? Cf::S_BYTES : 0));
          tma_load_3d(st, tX, &x_full[s], (h0 + k) * CK_P, s0, b);
          if (has_s)
            tma_load_2d(st + Cf::X_BYTES, &mp.S, &x_full[s], 0, (((b * nc + c) * p.heads) + h0 + k) * NS);
        };
        auto load_sc = [&](int k) {
          const int j = k % CK_SR;
          mbar_arrive_expect_tx(&sc_full[j], CK_SCAL * 4);
          bulk_load(sm + Cf::OFF_SC + j * CK_SCAL * 4, scal_bc + (int64_t)(h0 + k) * nc * CK_SCAL, CK_SCAL * 4,
                    &sc_full[j]);
        };
        mbar_arrive_expect_tx(cb_full, Cf::C_BYTES + Cf::KB * nk * 128);
        for (int a = 0; a < Cf::KAT; ++a) {
          tma_load_3d(sm + Cf::OFF_C + a * 128 * 128, &mp.C, cb_full, g * NS + a * 64, s0 + qb * 128, b);
          if (a < Cf::KB) tma_load_3d(sm + Cf::OFF_B + a * nk * 128, tB, cb_full, g * NS + a * 64, s0, b);
        }
        bool ok = true;
        if constexpr (Cf::KAT > Cf::KB) {  // the second half of B once the MMA has read the first
          ok = mbar_wait(b_free, 0, abort_flag);
          if (ok) {
            mbar_arrive_expect_tx(cb_full, (Cf::KAT - Cf::KB) * nk * 128);
            for (int a = Cf::KB; a < Cf::KAT; ++a)
              tma_load_3d(sm + Cf::OFF_B + (a - Cf::KB) * nk * 128, tB, cb_full, g * NS + a * 64, s0, b);
          }
        }
        // L2 prefetches SG_PF heads ahead of the loads: the stages alone hold too few bytes in flight
        // per SM to cover the memory latency
        auto prefetch = [&](int k) {
          tma_prefetch_3d(tX, (h0 + k) * CK_P, s0, b);
          if (has_s) tma_prefetch_2d(&mp.S, 0, (((b * nc + c) * p.heads) + h0 + k) * NS);
          if (has_z) tma_prefetch_3d(&mp.Z, (h0 + k) * CK_P, s0 + qb * 128, b);
          bulk_prefetch_l2(scal_bc + (int64_t)(h0 + k) * nc * CK_SCAL, CK_SCAL * 4);
        };
        for (int k = 1; k < min(SG_PF + 1, hcount); ++k) prefetch(k);
        for (int k = 0; k < min(CK_SR - 1, hcount); ++k) load_sc(k);
        load_xs(0);
        for (int k = 0; ok && k < hcount; ++k) {
          if (k + SG_PF + 1 < hcount) prefetch(k + SG_PF + 1);
          // x | S_in of head k+1 once the MMA of head k+1-STAGES has read its stage
          if (k + 1 < hcount) {
            const int prev = k + 1 - Cf::STAGES;
            const int ps = Cf::STAGES == 2 ? (prev & 1) : 0;
            const int pph = Cf::STAGES == 2 ? ((prev >> 1) & 1) : (prev & 1);
            if (prev >= 0 && !(ok = mbar_wait(&x_empty[ps], pph, abort_flag))) break;
            load_xs(k + 1);
          }
          // scalars of head k+3 into the slot head k-1 used
          if (k + CK_SR - 1 < hcount) {
            if (k >= 1 && !(ok = mbar_wait(&sc_free[(k - 1) % CK_SR], ((k - 1) / CK_SR) & 1, abort_flag))) break;
            load_sc(k + CK_SR - 1);
          }
        }
      }
    } else if (warp == 1) {
      // ------------------------------------------------ MMA issuer
      if (lane == 0) {
        constexpr int fmt = DT<T>::id == TH_BF16 ? 1 : 0;
        const uint32_t cA = smem_u32(sm + Cf::OFF_C), bA = smem_u32(sm + Cf::OFF_B);
        bool ok = mbar_wait(cb_full, 0, abort_flag);
        if (ok) {
          tc_fence_after();
          const uint32_t id_cb = make_idesc_f16(128, nk, fmt, 0, 0);
          for (int kk = 0; kk < NS / 16; ++kk) {
            if constexpr (Cf::KAT > Cf::KB) {
              if (kk == Cf::KB * 4) {  // d_state 256: the second half of B replaces the first
                tc_commit(b_free);
                if (!(ok = mbar_wait(cb_full, 1, abort_flag))) break;
                tc_fence_after();
              }
            }
            const int ba = (kk >> 2) & (Cf::KB - 1);
            const uint64_t ad = make_desc_sw128(cA + (kk >> 2) * 128 * 128 + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = make_desc_sw128(bA + ba * nk * 128 + (kk & 3) * 32, 16, 1024);
            tc_mma_f16(tmem, ad, bd, id_cb, kk ? 1u : 0u);
          }
          tc_commit(cb_done);
        }
        constexpr uint32_t id_y = make_idesc_f16(128, 64, fmt, 0, 1);  // B operand (x, S_in) MN-major
        int gu = 0;  // G units consumed
        for (int k = 0; ok && k < hcount; ++k) {
          const int xs = Cf::STAGES == 2 ? (k & 1) : 0;
          const int xph = Cf::STAGES == 2 ? ((k >> 1) & 1) : (k & 1);
          ok = mbar_wait(&x_full[xs], xph, abort_flag) && (k == 0 || mbar_wait(y_empty, (k - 1) & 1, abort_flag));
          if (!ok) break;
          const uint32_t xA = smem_u32(sm + Cf::OFF_X + xs * Cf::STAGE), sA = xA + Cf::X_BYTES;
          for (int un = 0; un < upk; ++un, ++gu) {
            const int slot = gu & 1;
            if (!(ok = mbar_wait(&g_full[slot], (gu >> 1) & 1, abort_flag))) break;
            tc_fence_after();
            for (int kk = 0; kk < 8; ++kk) {
              const uint32_t at = tmem + SG_T_G + slot * 64 + kk * 8;
              const uint64_t bd = make_desc_sw128(xA + (un * 8 + kk) * 2048, nk * 128, 1024);
              tc_mma_f16_ts(tmem + SG_T_Y, at, bd, id_y, (un | kk) ? 1u : 0u);
            }
            tc_commit(&g_free[slot]);
          }
          if (!ok) break;
          if (has_s) {
            for (int kk = 0; kk < NS / 16; ++kk) {
              const uint64_t ad = make_desc_sw128(cA + (kk >> 2) * 128 * 128 + (kk & 3) * 32, 16, 1024);
              const uint64_t bd = make_desc_sw128(sA + kk * 2048, NS * 128, 1024);
              tc_mma_f16(tmem + SG_T_Y + 64, ad, bd, id_y, kk ? 1u : 0u);
            }
          }
          tc_commit(&x_empty[xs]);
          tc_commit(y_full);
        }
      }
    } else if (warp < 2 + SG_BUILD_WARPS) {
      // ------------------------------------------------ G builders: four warps per TMEM lane quadrant,
      // each taking two of a unit's eight 16-key sub-blocks
      const int bw = warp - 2;
      const int q = warp & 3, part = bw >> 2;
      const int r = q * 32 + lane;      // row within the query half (TMEM lane)
      const int i = qb * 128 + r;       // row within the chunk
      const int R = qb * 128 + q * 32;  // first row of this warp
      const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
      bool ok = mbar_wait(cb_done, 0, abort_flag);
      int gu = 0;
      for (int k = 0; k < hcount; ++k) {
        const int j = k % CK_SR;
        ok = ok && mbar_wait(&sc_full[j], (k / CK_SR) & 1, abort_flag);
        const float* cum = reinterpret_cast<const float*>(sm + Cf::OFF_SC + j * CK_SCAL * 4);
        const float* dts = cum + CK_L;
        const float* colf = dts + CK_L;
        const float Dh = colf[CK_L];
        const float ci = cum[i];
        for (int un = 0; un < upk; ++un, ++gu) {
          const int slot = gu & 1;
          if (gu >= 2) ok = ok && mbar_wait(&g_free[slot], ((gu >> 1) - 1) & 1, abort_flag);
          ok = __all_sync(0xffffffffu, ok);
          if (ok) {
            tc_fence_after();
#pragma unroll
            for (int sb = 0; sb < 2; ++sb) {
              const int sub = part + 4 * sb;           // 16-key sub-block of the unit
              const int j0 = un * 128 + sub * 16;      // its first key
              const uint32_t gaddr = tl + SG_T_G + slot * 64 + sub * 8;
              uint32_t pk[8];
              if (j0 >= R + 32) {  // above every row of this warp: zeros
#pragma unroll
                for (int e = 0; e < 8; ++e) pk[e] = 0u;
                tmem_st8_nowait(gaddr, pk);
                continue;
              }
              uint32_t raw[16];
              tmem_ld16_issue(tl + j0, raw);
              // factors against the containing 32-key block's last column (the scalar record's colf):
              // exp(ci - cj) = exp(ci - c_ref) exp(c_ref - cj), neither of which can overflow below 80
              const float dref = ci - cum[j0 | 31];
              const bool fact = __all_sync(0xffffffffu, dref < 80.f);
              const float rf = __expf(fact ? dref : 0.f);
              tmem_wait_ld(raw);
              if (fact) {
                const uint64_t rf2 = f2_pack(rf, rf);
                const ulonglong2* cf = reinterpret_cast<const ulonglong2*>(colf + j0);  // 16-byte aligned
#pragma unroll
                for (int e4 = 0; e4 < 4; ++e4) {
                  const ulonglong2 c4 = cf[e4];
                  const uint64_t v01 =
                      f2_mul(f2_mul(rf2, c4.x), f2_pack(__uint_as_float(raw[4 * e4]), __uint_as_float(raw[4 * e4 + 1])));
                  const uint64_t v23 = f2_mul(f2_mul(rf2, c4.y),
                                              f2_pack(__uint_as_float(raw[4 * e4 + 2]), __uint_as_float(raw[4 * e4 + 3])));
                  float a0, a1, a2, a3;
                  f2_unpack(v01, a0, a1);
                  f2_unpack(v23, a2, a3);
                  raw[4 * e4] = __float_as_uint(a0);
                  raw[4 * e4 + 1] = __float_as_uint(a1);
                  raw[4 * e4 + 2] = __float_as_uint(a2);
                  raw[4 * e4 + 3] = __float_as_uint(a3);
                }
              } else {
                uint32_t tmp[16];  // the out-of-line call takes a copy: `raw` itself stays in registers
#pragma unroll
                for (int e = 0; e < 16; ++e) tmp[e] = raw[e];
                ssd_g_decay_slow(tmp, cum + j0, dts + j0, ci);
#pragma unroll
                for (int e = 0; e < 16; ++e) raw[e] = tmp[e];
              }
              if (j0 + 15 > R) {  // keys that may lie on or above the diagonal: causal mask and the D skip
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                  const int jj = j0 + e;
                  const float v = __uint_as_float(raw[e]);
                  raw[e] = __float_as_uint(jj < i ? v : (jj == i ? v + Dh : 0.f));
                }
              }
#pragma unroll
              for (int e2 = 0; e2 < 8; ++e2)
                pk[e2] = pack2<T>(__uint_as_float(raw[2 * e2]), __uint_as_float(raw[2 * e2 + 1]));
              tmem_st8_nowait(gaddr, pk);
            }
            tmem_wait_st();
            tc_fence_before();
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&g_full[slot]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sc_free[j]);
      }
    } else {
      // ------------------------------------------------ epilogue
      const int ew = warp - 2 - SG_BUILD_WARPS;
      const int q = warp & 3, half = ew >> 2;
      const int r = q * 32 + lane;
      const int i = qb * 128 + r;
      const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
      const int64_t trow = (int64_t)b * p.seq + s0 + i;
      const bool lead = ew == 0 && lane == 0;  // loads z and stores y
      auto tile = [&](int k) { return sm + Cf::OFF_ZY + (k & 3) * Cf::TILE; };
      auto fetch_z = [&](int k) {  // z of head k into its tile (or mark the free tile ready)
        if (has_z) {
          mbar_arrive_expect_tx(&z_full[k & 3], Cf::TILE);
          tma_load_3d(tile(k), &mp.Z, &z_full[k & 3], (h0 + k) * CK_P, s0 + qb * 128, b);
        } else {
          mbar_arrive(&z_full[k & 3]);
        }
      };
      bool ok = true;
      if (lead) {  // the tiles replace B: wait for the C.B^T MMA to have read it
        ok = mbar_wait(cb_done, 0, abort_flag);
        if (ok)
          for (int k = 0; k < min(4, hcount); ++k) fetch_z(k);
      }
      for (int k = 0; k < hcount; ++k) {
        const int j = k % CK_SR;
        // the tile of head k+2 reuses the one of head k-2 once that y has left (y of head k-1 may still
        // be in flight)
        if (lead && ok && k >= 2 && k + 2 < hcount) {
          bulk_wait_read1();
          fetch_z(k + 2);
        }
        ok = ok && mbar_wait(&sc_full[j], (k / CK_SR) & 1, abort_flag) &&
             mbar_wait(&z_full[k & 3], (k >> 2) & 1, abort_flag) && mbar_wait(y_full, k & 1, abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        float ss = 0.f;
        if (ok) {
          // y = (G.x + exp(cum_i) C.S_in) silu(z), 16 columns at a time straight out of TMEM; Y | Yo is
          // released as soon as the last columns are in registers
          const float* cum = reinterpret_cast<const float*>(sm + Cf::OFF_SC + j * CK_SCAL * 4);
          const float e = has_s ? __expf(cum[i]) : 0.f;
          uint8_t* yb = tile(k);  // holds z of this head (when gated); y is written in place
          tc_fence_after();
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t ry[16], ro[16];
            tmem_ld16_issue(tl + SG_T_Y + half * 32 + hh * 16, ry);
            if (has_s) tmem_ld16_issue(tl + SG_T_Y + 64 + half * 32 + hh * 16, ro);
            tmem_wait_ld(ry);
            tmem_wait_ld(ro);
            if (hh == 1) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(y_empty);
            }
#pragma unroll
            for (int c8 = 0; c8 < 2; ++c8) {
              T* at = reinterpret_cast<T*>(yb + sw128_off(r, half * 32 + hh * 16 + c8 * 8, 128));
              float zf[8], o[8];
              if (has_z) load8<T>(at, zf);
#pragma unroll
              for (int e8 = 0; e8 < 8; ++e8) {
                float y = __uint_as_float(ry[c8 * 8 + e8]);
                if (has_s) y = fmaf(e, __uint_as_float(ro[c8 * 8 + e8]), y);
                o[e8] = has_z ? y * silu_tanh(zf[e8]) : y;
              }
              ss += store8_ss<T>(at, o);  // sum of squares of the stored (rounded) values
            }
          }
          fence_proxy_async();
          red[(k & 1) * 256 + half * 128 + r] = ss;
        } else {
          __syncwarp();
          if (lane == 0) mbar_arrive(y_empty);
        }
        named_bar(2, 256);
        if (lead && ok) {
          tma_store_3d(&mp.Y, tile(k), (h0 + k) * CK_P, s0 + qb * 128, b);
          bulk_commit();
        }
        if (ok && half == 0 && i < len && p.gss)
          p.gss[trow * p.ldgss + h0 + k] = red[(k & 1) * 256 + r] + red[(k & 1) * 256 + 128 + r];
        __syncwarp();
        if (lane == 0) mbar_arrive(&sc_free[j]);
      }
      if (lead) bulk_wait0();
    }
    tc_fence_before();
    __syncthreads();  // this pass has drained: every store, load and MMA is complete
    tc_fence_after();
  }  // pass
  if (warp == 1) tmem_dealloc(tmem, 512);
}

template <typename T, int NS>
static int ssd_scan_launch(const ScMaps& m, const th_ssd_args* a, int nc, cudaStream_t st) {
  using Gf = SgCfg<NS>;
  if (int rc = smem_limit(ssd_scan_g<T, NS>, Gf::SMEM, "th_ssd(scan, G in TMEM)")) return rc;
  // head sets: about one CTA per SM
  const int hpg = a->heads / a->ngroups;
  const int per = a->batch * nc * a->ngroups;
  int nsets = per >= sm_count() ? 1 : sm_count() / per;
  nsets = nsets < 1 ? 1 : (nsets > hpg ? hpg : nsets);
  const int hs = (hpg + nsets - 1) / nsets;
  nsets = (hpg + hs - 1) / hs;
  const int units = per * nsets;
  launch_pdl(ssd_scan_g<T, NS>, dim3(units), dim3(SG_THREADS), Gf::SMEM, st, m, *a, nc, hs, nsets,
             reinterpret_cast<const float*>(a->workspace));
  return TH_OK;
}

// Applies to 2-byte dtypes with head_dim 64, state_dim 64, 128 or 256, chunk
// 256, 16-byte aligned rows, dt rows of a multiple of 4 floats and a large
// enough workspace; returns 1 (not taken) otherwise.  d_state 128 runs the
// chunk states as one serial walk per (batch, head); 64 and 256 run them
// chunk-parallel followed by the state pass.
template <typename T>
static int ssd_chunk_try(const th_ssd_args* a, cudaStream_t st, int* rc) {
  const int NS = a->state_dim;
  if (a->head_dim != CK_P || a->chunk != CK_L || (NS != 64 && NS != 128 && NS != 256)) return 1;
  if (!aligned16(a->x) || !aligned16(a->B) || !aligned16(a->C) || !aligned16(a->out) || !aligned16(a->dt) ||
      a->ldx % 8 || a->ldb % 8 || a->ldc % 8 || a->ldo % 8 || a->lddt % 4)
    return 1;
  if (a->z && (!aligned16(a->z) || a->ldz % 8)) return 1;
  if (!aligned16(a->workspace) || a->workspace_bytes < ck_ws_bytes(a->batch, a->seq, a->heads, NS)) return 1;
  const int nc = (a->seq + CK_L - 1) / CK_L;
  float* scal = reinterpret_cast<float*>(a->workspace);
  T* sin = reinterpret_cast<T*>(reinterpret_cast<uint8_t*>(a->workspace) + ck_scal_bytes(a->batch, a->heads, nc));
  T* sc = reinterpret_cast<T*>(reinterpret_cast<uint8_t*>(sin) + ck_state_bytes(a->batch, nc, a->heads, NS, CK_P));
  const uint64_t gw = (uint64_t)a->ngroups * NS, xw = (uint64_t)a->heads * CK_P;
  const uint64_t S = (uint64_t)a->seq, Bt = (uint64_t)a->batch;
  ScMaps m;
  CUtensorMap tdt;
  int r = make_tmap_3d(&m.B256, a->B, a->dtype, gw, S, Bt, a->ldb * 2, S * a->ldb * 2, 64, 256);
  if (!r) r = make_tmap_3d(&m.B128, a->B, a->dtype, gw, S, Bt, a->ldb * 2, S * a->ldb * 2, 64, 128);
  if (!r) r = make_tmap_3d(&m.C, a->C, a->dtype, gw, S, Bt, a->ldc * 2, S * a->ldc * 2, 64, 128);
  if (!r) r = make_tmap_3d(&m.X256, a->x, a->dtype, xw, S, Bt, a->ldx * 2, S * a->ldx * 2, 64, 256);
  if (!r) r = make_tmap_3d(&m.X128, a->x, a->dtype, xw, S, Bt, a->ldx * 2, S * a->ldx * 2, 64, 128);
  if (!r) r = make_tmap_3d(&m.Y, a->out, a->dtype, xw, S, Bt, a->ldo * 2, S * a->ldo * 2, 64, 128);
  m.Z = m.Y;
  if (!r && a->z) r = make_tmap_3d(&m.Z, a->z, a->dtype, xw, S, Bt, a->ldz * 2, S * a->ldz * 2, 64, 128);
  if (!r)
    r = make_tmap_2d(&m.S, sin, a->dtype, CK_P, (uint64_t)a->batch * nc * a->heads * NS, CK_P * 2, 64, NS, true);
  if (!r)
    r = make_tmap_3d(&tdt, a->dt, TH_F32, (uint64_t)a->heads, S, Bt, a->lddt * 4, S * a->lddt * 4, 4, 256, false);
  if (r) { *rc = r; return 0; }
  if ((*rc = smem_limit(ssd_state_tc<T>, StC::SMEM, "th_ssd(chunk states, tcgen05)"))) return 0;
  if ((*rc = smem_limit(ssd_chunk_states<T>, SpC::SMEM, "th_ssd(chunk states, parallel)"))) return 0;
  static const bool serial128 = [] {  // TH_SSD_STATES=p selects the parallel states for d_state 128 too
    const char* e = getenv("TH_SSD_STATES");
    return !(e && e[0] == 'p');
  }();
  if (NS == CK_NS && serial128) {
    launch_pdl(ssd_state_tc<T>, dim3((unsigned)a->heads, (unsigned)a->batch), dim3(320), StC::SMEM, st, m.B256, m.X256,
               tdt, m.S, *a, nc, scal);
    *rc = check_launch("th_ssd(chunk states, tcgen05)");
    if (*rc) return 0;
  } else {
    const int units = a->batch * nc * a->heads * ((NS + 127) / 128);
    const int grid = units < sm_count() ? units : sm_count();
    launch_pdl(ssd_chunk_states<T>, dim3(grid), dim3(320), SpC::SMEM, st, m.B256, m.X256, tdt, *a, nc, scal, sc);
    *rc = check_launch("th_ssd(chunk states, parallel)");
    if (*rc) return 0;
    if (nc > 1) {
      const int per = NS * CK_P / 4;
      launch_pdl(ssd_state_pass<T>, dim3((unsigned)((per + 255) / 256), (unsigned)a->heads, (unsigned)a->batch),
                 dim3(256), 0, st, *a, nc, (const float*)scal, (const T*)sc, sin);
      *rc = check_launch("th_ssd(state pass)");
      if (*rc) return 0;
    }
  }
  r = NS == 64 ? ssd_scan_launch<T, 64>(m, a, nc, st)
      : NS == 128 ? ssd_scan_launch<T, 128>(m, a, nc, st)
                  : ssd_scan_launch<T, 256>(m, a, nc, st);
  *rc = r ? r : check_launch("th_ssd(scan, tcgen05 multi-head)");
  return 0;
}

}  // namespace th
