/*
 * th_b200.h -- C ABI of the torch-helion B200 backend (libth_b200.so).
 *
 * The reference (ecolab-nus/torch-helion) lowers every partitioned OpIR
 * kernel to a generated Helion/Loom Python module
 * (src/torch_helion/codegen/emit.py:500-520, `emit_program`) and checks it
 * with a PyTorch interpreter (src/torch_helion/codegen/interpret.py:18-51,
 * `run_kernel`).  It has no native ABI of its own.  This header is the
 * boundary that replaces that seam: each entry point below executes one
 * OpIR `KernelSpec` kind (src/torch_helion/optimizer/opir.py:63-95) on an
 * sm_100a GPU.  The Python runtime (torch_helion.b200) binds it with ctypes.
 *
 * Conventions
 *   - Every pointer is a device pointer unless stated otherwise.  The caller
 *     owns all memory, outputs and workspaces included; nothing here calls
 *     cudaMalloc/cudaFree.  Workspace sizes come from th_*_workspace_size().
 *   - Matrices are row-major with an explicit leading dimension in
 *     ELEMENTS (`ld*`).  Activations are token-major [T, features],
 *     T = batch * seq, exactly the 2-D form the reference optimizer gives
 *     every activation (src/torch_helion/optimizer/passes.py:719-762).
 *   - Work is enqueued on `stream` (a cudaStream_t; NULL = legacy stream)
 *     on the CURRENT device.  Calls may come from several threads and for
 *     several devices in one process.  Process-wide state: a thread-local
 *     error string; one device-side error word per device (th_device_error);
 *     host caches guarded by mutexes -- encoded TMA descriptors (keyed by
 *     address and geometry), each kernel's raised shared-memory limit and the
 *     SM count (both per device ordinal), and th_ssd_noalloc's scratch
 *     address (per CUDA context).  None of it changes a call's result.
 *   - Return value: TH_OK (0) or a negative TH_E* code; the message is in
 *     th_last_error_string().
 */
#ifndef TH_B200_H_
#define TH_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status codes */
#define TH_OK 0
#define TH_EINVAL -1        /* bad shape / null pointer / bad enum          */
#define TH_EALIGN -2        /* pointer or leading dimension misaligned       */
#define TH_EDTYPE -3        /* dtype combination not supported               */
#define TH_ELAUNCH -4       /* CUDA launch or driver call failed             */
#define TH_ETIMEOUT -5      /* a device-side wait hit its iteration limit    */
#define TH_EUNSUPPORTED -6  /* valid request this build does not implement   */

/* ------------------------------------------------------------------ dtypes */
/* Mirrors the dtype names of the reference OpGraph TensorType
 * (src/torch_helion/capture/opgraph.py:26, DTYPE_BYTES). */
#define TH_F32 0
#define TH_BF16 1
#define TH_F16 2

/* ------------------------------------------------------------- activations */
#define TH_ACT_NONE 0
#define TH_ACT_SILU 1
#define TH_ACT_SOFTPLUS 2 /* log(1+exp(x)), identity above 20 as torch */
#define TH_ACT_GELU 3     /* 0.5 x (1 + erf(x / sqrt 2)), torch gelu(approximate='none') */
#define TH_ACT_GELU_TANH 4 /* torch gelu(approximate='tanh') */

/* ------------------------------------------------------------ housekeeping */
const char* th_last_error_string(void);
const char* th_version(void);
/* Reads (and with clear!=0 resets) the device error word that kernels set
 * when a bounded wait gives up.  Synchronises the current device. */
int th_device_error(int* out_code, int clear);

/* Diagnostic -- no counterpart in the reference (its kernels never run on a
 * device).  Launches one CTA whose thread 0 waits on an mbarrier through the
 * same bounded wait every pipelined kernel here uses, but with a limit of
 * `limit_ns`, while thread 32 arrives after `arrive_ns`.  *completed (device
 * memory) becomes 1 when the arrival was seen and 0 when the wait gave up,
 * in which case the device error word reports TH_DEVERR_MBAR_TIMEOUT (1)
 * through th_device_error.  limit_ns in [1e3, 1e8], arrive_ns in [0, 1e8]. */
int th_selftest_bounded_wait(int64_t limit_ns, int64_t arrive_ns, int32_t* completed, void* stream);

/* ----------------------------------------------------------------- rowstat
 * sumsq[r] = sum_k x[r,k]^2 (fp32).  Replaces the `row_sumsq` column the
 * reference keeps on a GEMM's K axis (passes.py:347-354, `_row_scale`;
 * partition.py:160-177 standalone norm kernel).  The GEMM epilogue turns it
 * into the RMSNorm row scale rsqrt(sumsq/K + eps). */
typedef struct {
  const void* x;
  int64_t ldx;
  float* sumsq; /* [rows] */
  int64_t rows, cols;
  int32_t dtype;
} th_rowstat_args;
int th_rowstat(const th_rowstat_args* a, void* stream);

/* ----------------------------------------------------------------- rmsnorm
 * y = x * rsqrt(mean(x^2) + eps) * gain -- the terminal norm kernel
 * (models/mamba.py:130-140, models/llama_block.py:55-63; reference lowering
 * passes.py:357-370 `_lower_standalone_rmsnorm`). */
typedef struct {
  const void* x;
  int64_t ldx;
  const float* gain; /* [cols] fp32, may be NULL (= ones) */
  void* y;
  int64_t ldy;
  int64_t rows, cols;
  float eps;
  int32_t dtype; /* dtype of x and y */
} th_rmsnorm_args;
int th_rmsnorm(const th_rmsnorm_args* a, void* stream);

/* ------------------------------------------------------------------- gemm
 * D[M, N] = epilogue(A[M, K] @ W[N, K]^T)
 * One kernel = one reference `gemm` KernelSpec: a shared LHS, sibling GEMMs
 * concatenated along N (partition.py:107-126), the RMSNorm sum-of-squares
 * fold (opir.py:13-20, `sumsq`) and an epilogue (interpret.py:22-35).
 * Epilogue stages, applied per element in this order:
 *   1. row scale:  acc *= rsqrt(sum_p rs_parts[r*rs_nparts+p]*rs_inv_k + rs_eps)
 *   2. column activation on [act_begin, act_end): acc = act(acc + bias[c-act_begin])
 *      (act TH_ACT_NONE with a bias: the bias alone)
 *   3. RoPE on [rope_begin, rope_end) (head_dim aligned): x*cos + rotate_half(x)*sin
 *      with position = row % rope_seq and fp32 tables [rope_seq, rope_head_dim]
 *   4. SwiGLU: W rows come in blocks of 128 = [64 gate | 64 up]; the output
 *      has N/2 columns, out = silu(gate) * up
 *   5. residual: out += residual[r, c]
 *   6. store in `dtype` (columns >= tail_begin go to out2 as fp32 instead)
 *   7. ss_out[r*ss_ld + c/64] = sum of squares of the stored values of the
 *      64-column group c/64 (feeds the next RMSNorm's row scale).
 * bf16/fp16 run on tcgen05 tensor cores (TMEM accumulators, TMA-fed smem
 * ring); fp32 runs an FFMA kernel so fp32 models keep fp32 accuracy. */
typedef struct {
  const void* a;
  int64_t lda;
  const void* w;
  int64_t ldw;
  void* d;
  int64_t ldd;
  int64_t m, n, k;
  int32_t dtype;
  /* 1. row scale */
  const float* rs_parts;
  int32_t rs_nparts;
  float rs_inv_k, rs_eps;
  /* 2. activation segment */
  int32_t act, act_begin, act_end;
  const float* bias;
  /* 3. rope */
  const float* rope_cos;
  const float* rope_sin;
  int32_t rope_begin, rope_end, rope_head_dim, rope_seq;
  /* 4. swiglu */
  int32_t swiglu;
  /* 5. residual (same dtype as d) */
  const void* residual;
  int64_t ld_res;
  /* 6. fp32 tail */
  float* out2;
  int64_t ld_out2;
  int32_t tail_begin; /* with out2: output columns >= tail_begin (>= 0) go to out2;
                         0 = all of them (d may then be NULL); >= n or no out2: no tail */
  /* 7. sum-of-squares partials of the stored output, one per 64 columns */
  float* ss_out;
  int64_t ss_ld;
  /* SMs the kernel's persistent grid may occupy (0 = all): leaves the rest to
   * work that runs beside it, e.g. a collective on another stream.  Such a
   * launch does not use programmatic dependent launch, so its CTAs do not
   * take the free SMs before the previous kernel of the stream ends. */
  int32_t sm_limit;
} th_gemm_args;
int th_gemm(const th_gemm_args* a, void* stream);

/* -------------------------------------------------------------- attention
 * Flash attention over token-major q/k/v views, the reference `attention`
 * kernel kind (opir.py:21-22; evaluate.py:139-146) extended with causal
 * masking and grouped-query heads (kv head = q head / (hq/hkv)).
 * q: [b*s, hq*d] at ldq, k/v: [b*s, hkv*d] at ldk/ldv, o: [b*s, hq*d]. */
typedef struct {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  int64_t ldq, ldk, ldv, ldo;
  int32_t batch, seq, hq, hkv, head_dim;
  float scale;
  int32_t causal;
  int32_t dtype;
} th_attention_args;
int th_attention(const th_attention_args* a, void* stream);

/* ---------------------------------------------------- causal conv1d + act
 * Depthwise causal conv over the sequence (models/mamba.py:278-283):
 * y[b,s,c] = act(sum_j w[c,j] * x[b, s-(width-1)+j, c]), zero left padding. */
typedef struct {
  const void* x;
  int64_t ldx;
  const float* w; /* [channels, width] fp32 */
  const float* bias; /* [channels] or NULL */
  void* y;
  int64_t ldy;
  int32_t batch, seq, channels, width;
  int32_t act;
  int32_t dtype;
} th_conv1d_args;
int th_conv1d(const th_conv1d_args* a, void* stream);

/* ------------------------------------------------------------ SSD (Mamba-2)
 * Chunked state-space-duality scan (models/mamba.py:163-223 `ssd_chunked`,
 * forward glue :297-327) with fp32 state:
 *   dA = dt*A, cumA = per-chunk inclusive cumsum of dA
 *   y  = sum_{j<=i in chunk} (C_i.B_j) exp(cumA_i-cumA_j) dt_j x_j
 *        + exp(cumA_i) C_i . S_in(chunk)  +  D*x_i
 *   S_in(c+1) = exp(cumA_last(c)) S_in(c) + sum_j exp(cumA_last-cumA_j) dt_j x_j B_j^T
 * Optional gate: out = y * silu(z) and gss[t*ngss + h] = sum_p out^2 (for the
 * gated RMSNorm that follows, mamba.py:327).
 * Heads share B/C in groups of hq/ngroups (ngroups=1: stock Mamba-2). */
typedef struct {
  const void* x;  int64_t ldx;  /* [T, h*p]                      */
  const float* dt; int64_t lddt; /* [T, h] fp32, softplus applied  */
  const float* A;                /* [h] fp32 (negative)            */
  const void* B;  int64_t ldb;  /* [T, g*n]                      */
  const void* C;  int64_t ldc;  /* [T, g*n]                      */
  const float* D;                /* [h] fp32 or NULL               */
  const void* z;  int64_t ldz;  /* [T, h*p] gate or NULL         */
  void* out;      int64_t ldo;  /* [T, h*p]                      */
  float* gss;     int64_t ldgss; /* [T, h] fp32 or NULL           */
  int32_t batch, seq, heads, head_dim, ngroups, state_dim, chunk;
  int32_t dtype;
  void* workspace;
  size_t workspace_bytes;
} th_ssd_args;
size_t th_ssd_workspace_size(int32_t batch, int32_t seq, int32_t heads, int32_t head_dim,
                             int32_t state_dim, int32_t chunk);
int th_ssd(const th_ssd_args* a, void* stream);

/* th_ssd_noalloc -- no counterpart in the reference.
 * The same scan as th_ssd for callers that cannot allocate device memory
 * where they call it (a host framework that keeps all device memory in its
 * own pool and forbids libraries from calling the CUDA allocator, a caller
 * that cannot afford the synchronisation a cudaFree implies, a plugin given
 * only input and output pointers).  `workspace`/`workspace_bytes` are
 * ignored: the chunk-state scratch is a file-scope device array of
 * TH_SSD_NOALLOC_MAX_BYTES that every GPU loading the library keeps until
 * exit; shapes needing more (see th_ssd_workspace_size) are rejected with
 * TH_EINVAL.  Inputs and outputs are still the caller's.  The first call in
 * a CUDA context looks up the array's device address with the caller's
 * device current (cudaGetSymbolAddress) and caches it per context (the
 * driver's context ID), so a device reset or another context on the same
 * device gets its own lookup; make that first call before any stream
 * capture.
 * All calls share the one array and it keeps the previous call's contents
 * (nothing in it needs to start at zero), so calls whose work overlaps on
 * the GPU -- concurrent streams, or threads sharing a device -- race. */
#define TH_SSD_NOALLOC_MAX_BYTES (32u << 20)
int th_ssd_noalloc(const th_ssd_args* a, void* stream);

/* -------------------------------------------------------------- embedding
 * out[t, :] = table[ids[t], :]  (aten.embedding capture, Mamba LM front). */
typedef struct {
  const int64_t* ids;
  const void* table;
  int64_t ldt;
  void* out;
  int64_t ldo;
  int64_t tokens, dim, vocab;
  int32_t dtype;
} th_embedding_args;
int th_embedding(const th_embedding_args* a, void* stream);

/* --------------------------------------------------------------- allreduce
 * In-place sum all-reduce of bytes [offset, offset + bytes) of a symmetric
 * buffer across `world` ranks on one NVSwitch node, through the switch's
 * multicast (multimem.ld_reduce / multimem.st; NVLS).  Replaces the NCCL
 * all-reduce the tensor-parallel Llama block runs after its row-split
 * projections (the reference has no multi-GPU path; the exchange itself is
 * the standard Megatron split: o_proj and down_proj partial sums).
 *
 * Every rank calls it with the same offset, bytes, dtype and ctas, in the
 * same order (like any collective), each on its own GPU.  Rank r reduces
 * slice r (bytes / world) of the range and writes the sum to every rank.
 * `sig` is this rank's TH_ALLREDUCE_SIGNAL_BYTES signal pad (zeroed once
 * before the first call, on every rank, before any rank calls), `peer_sig` a
 * device array of `world` pointers to every rank's pad as mapped in this
 * process.  bf16 / f16 are summed with fp32 accumulation.  bytes must be a
 * multiple of 16 x world; `mc + offset` and `sig` 16-byte aligned.  The
 * handshakes wait at most 2 s: then the device error word reports
 * TH_DEVERR_MBAR_TIMEOUT and the range is left partly reduced.  ctas: grid
 * size (0 = 32, at most TH_ALLREDUCE_MAX_CTAS); every rank must pass the same
 * value.  world == 1 returns at once. */
#define TH_ALLREDUCE_MAX_CTAS 256
#define TH_ALLREDUCE_MAX_WORLD 8
#define TH_ALLREDUCE_SIGNAL_BYTES 20480
typedef struct {
  void* mc;               /* multicast address of the buffer (offset 0) */
  void* const* peer_sig;  /* device array [world] of signal-pad pointers */
  void* sig;              /* this rank's signal pad */
  int64_t offset, bytes;
  int32_t dtype, rank, world, ctas;
  /* optional row statistics: when sumsq_mc (the multicast address of an fp32
   * array in symmetric memory, element i = row i of the buffer) is set, every
   * rank's slice must be whole rows of row_bytes bytes (offset and bytes
   * multiples of row_bytes, bytes of row_bytes x world); each reduced row's
   * sum of squares (fp32) is stored to element row of every rank's array */
  float* sumsq_mc;
  int64_t row_bytes;
} th_allreduce_args;
int th_allreduce(const th_allreduce_args* a, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TH_B200_H_ */
