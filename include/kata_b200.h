/*
 * kata_b200.h -- C ABI of the B200 (sm_100a) KATA-SPD attention hot path.
 *
 * This is the drop-in boundary below the reference's Python operator API.  Each entry point
 * takes plain device pointers, sizes and a CUDA stream; no PyTorch (or other framework) type
 * appears in any signature.  The library never allocates or frees device memory: outputs and
 * workspace are owned by the caller, and no pointer is retained after a call returns.  Every
 * call is stream-ordered on the given stream and performs no host synchronisation.
 *
 * Layout: all token tensors are time-major and contiguous, i.e. (B, T, heads, dim) with dim
 * fastest, exactly as the reference launchers require after their .contiguous() calls
 * (kata/parallel_kata_attn.py:229-231).  Per-token scalars (den, c, beta, gates) are (B, T, heads).
 *
 * Return value: KATA_OK (0) or a negative KATA_ERR_* code; kata_strerror() names it.
 * Device-side bounded waits never trap: when one times out the kernel stores a nonzero code
 * into *status (if status != NULL) and returns early.  Callers check the word after the stream
 * drains (KATA_STATUS_* values).
 */
#ifndef KATA_B200_H
#define KATA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define KATA_API __attribute__((visibility("default")))
#else
#define KATA_API
#endif

/* Same object as cudaStream_t / CUstream; declared opaquely so this header needs no CUDA. */
typedef struct CUstream_st* kata_stream_t;

enum {
  KATA_OK = 0,
  KATA_ERR_INVALID = -1,     /* null pointer or inconsistent argument */
  KATA_ERR_DTYPE = -2,       /* unsupported dtype */
  KATA_ERR_SHAPE = -3,       /* unsupported or inconsistent shape */
  KATA_ERR_ALIGN = -4,       /* pointer not 16-byte aligned (TMA requirement) */
  KATA_ERR_WORKSPACE = -5,   /* workspace missing or too small */
  KATA_ERR_CUDA = -6,        /* a CUDA runtime call failed (e.g. launch error) */
  KATA_ERR_DRIVER = -7,      /* driver entry point (tensor-map encoder) unavailable */
  KATA_ERR_UNSUPPORTED = -8, /* algorithm not available for this configuration */
  KATA_ERR_SCRATCH_LIMIT = -9 /* problem needs more scratch than the library's fixed array */
};

/* Values a kernel may store into the optional device status word. */
enum { KATA_STATUS_OK = 0, KATA_STATUS_WAIT_TIMEOUT = 1 };

enum { KATA_DTYPE_F32 = 0, KATA_DTYPE_BF16 = 1, KATA_DTYPE_F16 = 2 };

/* Kernel family.  AUTO picks the tcgen05 tensor-core kernels for bf16/f16 inputs whose shape
 * they cover and the fp32-exact SIMT kernels otherwise (fp32 inputs always take SIMT, which is
 * the fp32-accurate mode).  TC / SIMT force one family (TC returns KATA_ERR_UNSUPPORTED when the
 * shape or dtype is outside its envelope).
 * TC_GRAM: the sum score with groups of 16 (D = 16 M, D in {64, 128}, Dv = 64, bf16) as a linear
 * score over the 136 entries of the group Gram matrix G(x) = sum_a x_a x_a^T (A[t,s] =
 * scale^2 <G(q_t), G(k_s)>, the same function): one K = 144 tensor-core product per score tile
 * instead of M^2 squared parts.  It needs a workspace (kata_attn_fwd_workspace_bytes /
 * kata_attn_bwd_workspace_bytes); AUTO takes it for such problems when the workspace passed is at
 * least that large, and the parts form (TC) otherwise.  No counterpart in the reference, whose sum
 * kernels square the M^2 parts. */
enum { KATA_ALGO_AUTO = 0, KATA_ALGO_TC = 1, KATA_ALGO_SIMT = 2, KATA_ALGO_TC_GRAM = 3 };

/* Score form.  CONCAT: A[t,s] = sum_g (scale * q_g[t].k_g[s])^2  (kata_quadratic)
 *              SUM:    A[t,s] = sum_{i,j} (scale * q_i[t].k_j[s])^2 (kata_quadratic_sum) */
enum { KATA_SCORE_CONCAT = 0, KATA_SCORE_SUM = 1 };

/* ---------------------------------------------------------------------------------------------
 * Causal normalised KATA-SPD attention, forward.
 *   o_t = sum_{s<=t} A[t,s] v_s / den_t,  den_t = sum_{s<=t} A[t,s]  (den_t <= 0 -> divide by 1)
 *   with A optionally multiplied by exp(min(c_t - c_s, 0)) when c != NULL.
 * Replaces the Triton launchers parallel_kata_attn_fwd_impl (kata/parallel_kata_attn.py:211-288)
 * and parallel_kata_attn_sum_fwd_impl (kata/parallel_kata_attn.py:539-576), i.e. kernels
 * parallel_kata_attn_fwd_kernel (kata/kernels/parallel_kata.py:10-197) and
 * parallel_kata_attn_sum_fwd_kernel (kata/kernels/parallel_kata.py:202-345).
 * GQA: HQ must be a multiple of H; query head hq reads key/value head hq / (HQ/H).
 * ------------------------------------------------------------------------------------------- */
typedef struct {
  const void* q;   /* (B,T,HQ,D)  dtype                                  */
  const void* k;   /* (B,T,H,D)   dtype                                  */
  const void* v;   /* (B,T,H,Dv)  dtype                                  */
  const float* c;  /* (B,T,HQ) fp32 cumulative log-decay, or NULL         */
  void* o;         /* (B,T,HQ,Dv) dtype   [out]                          */
  float* den;      /* (B,T,HQ) fp32       [out]                          */
  int* status;     /* optional device status word (int32), may be NULL   */
  int dtype;       /* KATA_DTYPE_*                                       */
  int B, T, H, HQ, D, Dv;
  int M;           /* num_groups; D % M == 0                             */
  int score;       /* KATA_SCORE_*                                       */
  int algo;        /* KATA_ALGO_*                                        */
  float scale;     /* per-group dot scale (reference default 1/sqrt(D/M)) */
  void* workspace; /* optional: kata_attn_fwd_workspace_bytes(args) bytes, 16-byte aligned
                      (TC_GRAM only; NULL / 0 -> AUTO runs the parts form) */
  size_t workspace_bytes;
  const int* cu_seqlens; /* optional packed documents: (num_seqs + 1) int32 device offsets into T,
                            0 = cu[0] <= cu[1] <= ... <= cu[num_seqs] = T, with B = 1; token t of
                            document n attends to the tokens s <= t of document n only (the kernels
                            clamp the offsets into [0, T] and to non-decreasing order, so a malformed
                            array gives wrong documents but no out-of-bounds access).  Tensor-core
                            parts form only (bf16 / f16; decay allowed, c per packed token):
                            KATA_ERR_UNSUPPORTED otherwise */
  int num_seqs;
} kata_attn_fwd_args;

KATA_API int kata_attn_fwd(const kata_attn_fwd_args* args, kata_stream_t stream);
/* Device workspace the forward can use: the bf16 Gram features of q and k when TC_GRAM (or AUTO
 * on a TC_GRAM problem) applies, else 0. */
KATA_API size_t kata_attn_fwd_workspace_bytes(const kata_attn_fwd_args* args);

/* Kernel family that kata_attn_fwd / kata_attn_bwd would run for these arguments with the workspace
 * that kata_attn_*_workspace_bytes asks for (only the shape, dtype, score, decay and algo fields
 * are read; no pointer is touched): KATA_ALGO_TC_GRAM or KATA_ALGO_TC (tcgen05) or KATA_ALGO_SIMT
 * (fp32 CUDA cores), or a negative KATA_ERR_* code.  Lets a binding tell a caller
 * when a bf16/f16 problem falls outside the tensor-core envelope and runs on the much slower SIMT
 * kernels.  No counterpart in the reference (its Triton kernels have a single path). */
KATA_API int kata_attn_algo(const kata_attn_fwd_args* args);

/* ---------------------------------------------------------------------------------------------
 * Causal normalised KATA-SPD attention, backward.
 *   delta_t = <o_t, dO_t>;  dA[t,s] = (dO_t.v_s - delta_t) / den_t  (causal);
 *   dq, dk from d(qk_p) = 2 qk_p dA (times the decay factor); dv = (A/den)^T dO;
 *   dc_t = sum_s G[t,s] - sum_t' G[t',t], G = dA * A over pairs with c_t - c_s <= 0.
 * Replaces parallel_kata_attn_bwd_triton (kata/parallel_kata_attn.py:364-529) with kernels
 * K3-K9 (kata/kernels/parallel_kata.py:349-1342), the sum-form Triton backward
 * (kata/parallel_kata_attn.py:755-901, kata/kernels/parallel_kata_sum.py), the PyTorch
 * fallbacks parallel_kata_attn_bwd (:49-146) / parallel_kata_attn_bwd_sum_torch (:579-653),
 * and the autograd recompute of the decayed form (_KataDecayFunction.backward, :329-347).
 * workspace: kata_attn_bwd_workspace_bytes(args) bytes of device memory (may be 0 -> NULL ok);
 * the size depends on B, T, HQ and on whether c is given (decay adds a head-major copy of c), and
 * on a TC_GRAM problem (algo AUTO or TC_GRAM) it adds the Gram features and their gradients.  AUTO
 * given less than that, but at least the parts-form size, runs the parts form.
 * ------------------------------------------------------------------------------------------- */
typedef struct {
  const void* q;     /* (B,T,HQ,D)  dtype */
  const void* k;     /* (B,T,H,D)   dtype */
  const void* v;     /* (B,T,H,Dv)  dtype */
  const void* o;     /* (B,T,HQ,Dv) dtype (forward output) */
  const float* den;  /* (B,T,HQ) fp32 (forward denominator) */
  const void* dout;  /* (B,T,HQ,Dv) dtype, upstream gradient */
  const float* c;    /* (B,T,HQ) fp32 or NULL */
  void* dq;          /* (B,T,HQ,D)  dtype [out] */
  void* dk;          /* (B,T,H,D)   dtype [out] */
  void* dv;          /* (B,T,H,Dv)  dtype [out] */
  float* dc;         /* (B,T,HQ) fp32 [out], required iff c != NULL */
  void* workspace;
  size_t workspace_bytes;
  int* status;
  int dtype;
  int B, T, H, HQ, D, Dv;
  int M;
  int score;
  int algo;
  float scale;
  int phases;        /* 0 = full backward; 1 = dq pass only (also fills the workspace: delta,
                        1/den, delta/den, dc row part); 2 = dk/dv pass only (needs a prior dq
                        pass on the same workspace).  Splitting lets a caller time each pass. */
  const int* cu_seqlens; /* optional packed documents, as in kata_attn_fwd_args (the workspace
                            size depends on num_seqs) */
  int num_seqs;
} kata_attn_bwd_args;

KATA_API size_t kata_attn_bwd_workspace_bytes(const kata_attn_bwd_args* args);
KATA_API int kata_attn_bwd(const kata_attn_bwd_args* args, kata_stream_t stream);

/* Backward for callers that cannot allocate device memory.  No counterpart in the reference.
 * Some callers cannot call cudaMalloc: host code that runs under a fixed, pre-reserved device
 * memory budget that forbids further allocation once loaded, or a plugin host whose operator
 * interface passes the kernel only its inputs and outputs and offers no workspace.  This entry
 * point runs exactly the computation of kata_attn_bwd but ignores args->workspace and uses a
 * 16 MiB file-scope device array of the library instead (held on every GPU that loads the
 * library until the process exits).  Problems whose parts-form workspace
 * (kata_attn_bwd_workspace_bytes() with algo TC or SIMT; TC_GRAM's own size for algo TC_GRAM)
 * exceeds 16 MiB are rejected with KATA_ERR_SCRATCH_LIMIT; AUTO runs the Gram form of a sum-score
 * problem only when its larger workspace fits in the array.  The first call on a device resolves the
 * array's address for that device, so make it outside any stream capture; the address is kept for
 * the life of the process, so the device must not be reset (cudaDeviceReset) between calls.  All
 * calls on a device share the array: calls whose kernels overlap on the GPU race on it.  Only the
 * full backward is accepted (phases must be 0; 1 and 2 return KATA_ERR_INVALID), because a
 * dk/dv-only pass would read whatever the previous call on the device left in the shared array.
 * The caller still passes every input and output buffer; this path calls no allocating routine. */
KATA_API int kata_attn_bwd_noalloc(const kata_attn_bwd_args* args, kata_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * SPD delta rule (DeltaKATA), forward.
 *   kappa(x,y) = sum_{g,h} (scale * x_g . y_h)^2   over all M*M group pairs (E = D/M)
 *   U = (I + diag(beta) tril(kappa(k,k), -1))^{-1} diag(beta) v
 *   num = tril(kappa(q,k)) U (diagonal included),  den_t = sum_{s<=t} kappa(q_t,k_s)
 *   o = num / (den + eps) if normalize else num
 * Replaces flash_delta_U (kata/spd/flash_delta.py:186-212, kernel K14 :27-183),
 * flash_delta_readout (:975-983, K15 :900-972) and flash_delta_den (:1049-1057, K16 :988-1046),
 * i.e. _FlashDelta.forward (:1062-1081).  The reference requires T % 64 == 0; any T >= 1 works here.
 * kappa is the attention "sum" score, so the readout runs on the attention kernels (tensor cores for
 * bf16/fp16), and U comes from an O(T) chunk scan over the E^2-feature state sum psi(k) U^T
 * (psi(x)[a,b] = scale sum_g x_{g,a} x_{g,b}) instead of the reference's O(T^2) chunk loop.
 * Supported: M <= 4, D/M a multiple of 8 with (D/M)^2 <= 4096, D <= 256, Dv a multiple of 16 <= 256.
 * Outputs are fp32 like the reference's.  E = tril(kappa(k,k),-1) U (the erase term) is written
 * when E != NULL.  phases: 0 = U (+E) then o and den; 1 = U (+E) only (flash_delta_U);
 * 2 = readout from a given U: o when o != NULL (flash_delta_readout), den when den != NULL
 * (flash_delta_den; U may then be NULL); v, beta, E unused.
 * ------------------------------------------------------------------------------------------- */
typedef struct {
  const void* q;     /* (B,T,H,D)  dtype */
  const void* k;     /* (B,T,H,D)  dtype */
  const void* v;     /* (B,T,H,Dv) dtype */
  const float* beta; /* (B,T,H) fp32 */
  float* U;          /* (B,T,H,Dv) fp32 [out; in for phases == 2] */
  float* E;          /* (B,T,H,Dv) fp32 [out] or NULL */
  float* o;          /* (B,T,H,Dv) fp32 [out] */
  float* den;        /* (B,T,H) fp32 [out] (written for both normalize settings) */
  int dtype;         /* of q, k, v */
  int B, T, H, D, Dv;
  int M;             /* groups; D % M == 0, M*M <= 16 */
  int normalize;
  float scale;       /* reference default 1/E */
  float eps;
  int phases;
  void* workspace;           /* kata_delta_fwd_workspace_bytes(args) bytes of device memory */
  size_t workspace_bytes;
  float* state;              /* (B,H,E*E,Dv) fp32 [out] or NULL: the final state sum_t psi(k_t) U_t^T with
                                psi(x)[a,b] = scale sum_g x_{g,a} x_{g,b} (flash_delta_state's S) */
} kata_delta_fwd_args;

KATA_API size_t kata_delta_fwd_workspace_bytes(const kata_delta_fwd_args* args);
KATA_API int kata_delta_fwd(const kata_delta_fwd_args* args, kata_stream_t stream);

/* SPD delta rule, backward: dq, dk, dv, dbeta (fp32) from the forward's U (and o, den) and dO.
 * normalize: dO' = dO/(den+eps) and z_t = <dO_t,o_t>/(den_t+eps) enter dA_qk = dO'.U - z
 * (the "consistent" normalised backward, kata/spd/flash_delta.py:1084-1108).
 * z != NULL selects the reference's flash_delta_bwd(..., do, z) contract instead: dout is the
 * already-scaled dO' and z the centring term; o, den and normalize are then unused.
 * E == NULL: the erase term is recomputed into the workspace (as the reference does).
 * Replaces flash_delta_bwd (kata/spd/flash_delta.py:830-895) with K17-K21 (:267-827). */
typedef struct {
  const void* q;
  const void* k;
  const void* v;
  const float* beta;
  const float* U;
  const float* E;    /* or NULL */
  const float* o;
  const float* den;
  const float* dout; /* (B,T,H,Dv) fp32 */
  const float* z;    /* (B,T,H) fp32 or NULL */
  float* dq;         /* (B,T,H,D) fp32 [out] */
  float* dk;         /* (B,T,H,D) fp32 [out] */
  float* dv;         /* (B,T,H,Dv) fp32 [out] */
  float* dbeta;      /* (B,T,H) fp32 [out] */
  void* workspace;
  size_t workspace_bytes;
  int dtype;
  int B, T, H, D, Dv;
  int M;
  int normalize;
  float scale;
  float eps;
} kata_delta_bwd_args;

KATA_API size_t kata_delta_bwd_workspace_bytes(const kata_delta_bwd_args* args);
KATA_API int kata_delta_bwd(const kata_delta_bwd_args* args, kata_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Gated delta rule (GDN), forward: per (sequence, value head), for t in order
 *   S <- exp(g_t) S;  u_t = beta_t (v_t - S^T k_t);  S <- S + k_t u_t^T;  o_t = scale S^T q_t
 * computed chunk-wise (64 tokens) in the WY form.  Replaces fla's chunk_gated_delta_rule_fwd
 * (fla/ops/gated_delta_rule/chunk.py:29-114, the arithmetic of chunk_gated_delta_rule :365-526),
 * which the reference calls for its gated_deltanet models; fla is third-party (pinned 0.5.0,
 * scripts/setup.sh:27).  Token tensors are time-major; with cu_seqlens (B == 1) the tokens of
 * sequence n are [cu_seqlens[n], cu_seqlens[n+1]) and chunk_offsets[n] is the index of its first
 * 64-token chunk (chunk_offsets[N] == num_chunks).  Without cu_seqlens N == B and
 * num_chunks == B * ceil(T/64).  This build covers K == V == 64.
 * A receives, per token row, its row of the chunk's (I + L)^{-1} (fla's A); the backward takes it.
 * ------------------------------------------------------------------------------------------- */
typedef struct {
  const void* q;             /* (B,T,H,K)  dtype */
  const void* k;             /* (B,T,H,K)  dtype */
  const void* v;             /* (B,T,HV,V) dtype */
  const float* g;            /* (B,T,HV) per-token log gate (not cumulated) */
  const float* beta;         /* (B,T,HV) */
  const float* h0;           /* (N,HV,K,V) initial state or NULL */
  void* o;                   /* (B,T,HV,V) dtype [out] */
  float* ht;                 /* (N,HV,K,V) final state [out] or NULL */
  float* A;                  /* (B,T,HV,64) [out] */
  const int* cu_seqlens;     /* (N+1) int32 device or NULL */
  const int* chunk_offsets;  /* (N+1) int32 device or NULL (iff cu_seqlens is NULL) */
  void* workspace;
  size_t workspace_bytes;
  int dtype;
  int B, T, H, HV, K, V;
  int N, num_chunks;
  float scale;               /* fla default K^-0.5 */
  int algo;                  /* KATA_ALGO_*: AUTO = tcgen05 kernels for bf16/f16 inputs, fp32-exact CUDA-core
                                kernels for fp32 inputs; TC / SIMT force one (TC needs 16-bit inputs) */
} kata_gdn_fwd_args;

KATA_API size_t kata_gdn_fwd_workspace_bytes(const kata_gdn_fwd_args* args);
KATA_API int kata_gdn_fwd(const kata_gdn_fwd_args* args, kata_stream_t stream);

/* Gated delta rule, backward: dq, dk (per q/k head, summed over its value heads), dv, dg (per-token
 * log gate), dbeta, dh0, all fp32, from the forward's inputs, its A and dO (+ d final state).
 * Replaces fla's chunk_gated_delta_rule_bwd (fla/ops/gated_delta_rule/chunk.py:117-236). */
typedef struct {
  const void* q;
  const void* k;
  const void* v;
  const float* g;
  const float* beta;
  const float* h0;           /* or NULL */
  const float* A;            /* the forward's A */
  const void* dout;          /* (B,T,HV,V) dtype */
  const float* dht;          /* (N,HV,K,V) or NULL */
  void* dq;                  /* (B,T,H,K) [out], fp32 or grad_dtype */
  void* dk;                  /* (B,T,H,K) [out] */
  void* dv;                  /* (B,T,HV,V) [out] */
  float* dg;                 /* (B,T,HV) [out] */
  float* dbeta;              /* (B,T,HV) [out] */
  float* dh0;                /* (N,HV,K,V) [out] or NULL */
  const int* cu_seqlens;
  const int* chunk_offsets;
  void* workspace;
  size_t workspace_bytes;
  const void* fwd_workspace; /* the forward call's workspace, unchanged since, or NULL: with it the
                                backward reuses the forward's chunk states instead of recomputing
                                them (and needs a smaller workspace) */
  int dtype;
  int B, T, H, HV, K, V;
  int N, num_chunks;
  float scale;
  int algo;                  /* KATA_ALGO_*, as in the forward; the backward must use the forward's family
                                when fwd_workspace is given (the two families lay the workspace out differently) */
  int grad_dtype;            /* KATA_DTYPE_F32 (0): dq, dk, dv are fp32.  The input dtype: dq, dk, dv are written
                                in it (tensor-core family with H == HV only, else KATA_ERR_UNSUPPORTED); dg,
                                dbeta, dh0 stay fp32 */
} kata_gdn_bwd_args;

KATA_API size_t kata_gdn_bwd_workspace_bytes(const kata_gdn_bwd_args* args);
KATA_API int kata_gdn_bwd(const kata_gdn_bwd_args* args, kata_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Sequence-parallel KATA-SPD (concat score) building blocks.  No counterpart in the reference (its
 * "parallel" means parallel over T inside one GPU); they implement the cross-shard prefix of a
 * sequence split contiguously across ranks.  With psi(x)[g,a,b] = scale * x_{g,a} x_{g,b}
 * (F = M E^2 features), A[t,s] = psi(q_t).psi(k_s); earlier shards contribute psi(q_t)^T P with
 * P = sum_s psi(k_s) [v_s | 1].  Feature tensors are head-major (B,H,T,F) bf16.
 * ------------------------------------------------------------------------------------------- */
/* R = psi(x) for x (B,T,H,D) of `dtype`; (D/M) % 8 == 0; R 16-byte aligned. */
KATA_API int kata_sp_features(const void* x, void* R, int dtype, int B, int T, int H, int D, int M, float scale,
                              kata_stream_t stream);
/* R = psi_sum(x), the sum score's features psi[a,b] = scale * sum_g x_{g,a} x_{g,b} (F = E^2), for x
 * (B,T,H,D) of `dtype`, R (B,H,T,F) bf16; (D/M) % 8 == 0; R 16-byte aligned.  Used for the state of
 * the sum score's decode path (the reference's parallel_kata_attn_sum score, kata/parallel_kata_attn.py:737). */
KATA_API int kata_sum_features(const void* x, void* R, int dtype, int B, int T, int H, int D, int M, float scale,
                               kata_stream_t stream);
/* dx (B,T,H,D) fp32 (+)= factor * sum_b G[g,b,a] x_{g,b}: the gradient of psi for a feature
 * gradient G (B,H,T,F) bf16 that is symmetric in (a,b) (factor = 2 * scale). */
KATA_API int kata_sp_contract(const void* G, const void* x, float* dx, int dtype, int B, int T, int H, int D, int M,
                              float factor, int accumulate, kata_stream_t stream);
/* o = (o_local * den_local' + X) / D',  D = den_local + y  (z' = z if z > 0 else 1), where
 * XY (B,H,T,ldxy) fp32 holds X in columns [0,Dv) and y in column Dv; o_local, o (B,T,H,Dv) dtype,
 * den_local, D (B,T,H) fp32. */
KATA_API int kata_sp_combine(const void* o_local, const float* den_local, const float* XY, void* o, float* D_out,
                             int dtype, int B, int T, int H, int Dv, int ldxy, kata_stream_t stream);
/* W1 (B,H,T,ldw) bf16 = [dO/D' | -<dO,o>/D' | 0 ...] for o, dO (B,T,H,Dv) dtype and D (B,T,H). */
KATA_API int kata_sp_bwd_prep(const void* o, const void* dout, const float* D_in, void* W1, int dtype, int B, int T,
                              int H, int Dv, int ldw, kata_stream_t stream);

/* Quadratic-feature contractions on the tensor cores, psi formed in shared memory (never written to
 * global memory) as the bf16 rounding of the unscaled products x_a x_b (sum score: of the fp32 sum over
 * groups), the scale multiplying the fp32 result.  psi is the concat map above (F = M E^2), or for
 * score == KATA_SCORE_SUM in
 * kata_sp_state the sum map psi[a,b] = scale sum_g x_{g,a} x_{g,b} (F = E^2).  x is a (B,T,H,D) 16-bit
 * token tensor (q or k) with E = D / M in {16, 32} and D in {64, 128} (sum score: M <= 4); W is
 * (B*H, T, ldw) bf16 and P^T (B*H, ldw, F) bf16, ldw a multiple of 8, <= 144.  All pointers 16-byte
 * aligned.  No counterpart in the reference (these replace GEMMs on a materialised psi).
 *   kata_sp_state:  S[f, n] = sum_t psi(x_t)[f] W[t, n] for W of H*G heads (W head w reads x head w / G),
 *                   stored as S^T (B*H*G, ldw, F) fp32 (trans = 1) or S (B*H*G, F, lds) fp32 (trans = 0;
 *                   columns ldw..lds-1 zeroed, lds % 4 == 0)
 *   kata_sp_apply:  Y[t, n] = sum_f psi(x_t)[f] P[f, n] for x of H heads and P of H/G heads (x head h reads
 *                   P head h / G); dv_mode 0 stores Y (B*H, T, ldw) fp32, dv_mode 1 adds Y[:, :Dv] into
 *                   dv (B,T,H,Dv) fp32 (passed as Y)
 *   kata_sp_grad:   dx[t, g E + a] += factor * sum_b (W P^T)[t, (g,a,b)] x[t, g E + b]  (dx (B,T,H,D)
 *                   fp32; for a P symmetric in (a, b) and factor = 2 scale this is the gradient of psi)
 * status is the optional device status word (may be NULL) that a timed-out wait writes. */
KATA_API int kata_sp_state(const void* x, const void* W, float* S, int dtype, int B, int T, int H, int G, int D,
                           int M, int score, int ldw, float scale, int trans, int lds, int* status,
                           kata_stream_t stream);
KATA_API int kata_sp_apply(const void* x, const void* P, float* Y, int dtype, int B, int T, int H, int G, int D,
                           int M, int ldw, float scale, int dv_mode, int Dv, int* status, kata_stream_t stream);
KATA_API int kata_sp_grad(const void* W, const void* P, const void* x, float* dx, int dtype, int B, int T, int H,
                          int D, int M, int ldw, float factor, int* status, kata_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Decode (generation) step of KATA-SPD attention.  No counterpart in the reference: its
 * quadratic-feature branch keeps no recurrent state (kata/layer.py:421-492 sets final_state = None;
 * :532-537 caches it), so each generated token re-runs causal attention over the whole prefix.
 * Both scores are psi(q).psi(k) for quadratic features psi (E = D/M):
 *   concat  psi(x)[g,a,b] = scale x_{g,a} x_{g,b}        F = M E^2
 *   sum     psi(x)[a,b]   = scale sum_g x_{g,a} x_{g,b}  F = E^2
 * The state of a prefix is S = sum_s w_s psi(k_s) [v_s | 1], (B*HS, F, lds) fp32: columns [0,Dv)
 * the weighted value sums, column Dv the weighted key-feature sum, columns above Dv zero
 * (lds % 4 == 0, Dv + 1 <= lds <= 1024).  Without decay (g == NULL) w_s = 1 and there is one state
 * per key/value head (HS = H), shared by its HQ/H in {1,2,4,8} query heads.  With decay, g (B,HQ)
 * fp32 is the token's log-decay c_t - c_{t-1}, w_s = exp(c_t - c_s), and the state is per query
 * head (HS = HQ); this equals the reference's exp(min(c_t - c_s, 0)) whenever c is non-increasing,
 * as the layer's c = cumsum(-exp(A_log) softplus(dt)) is (kata/layer.py:440-447).  One call takes
 * one new token per (batch, head):
 *   S = exp(g) S + psi(k) [v | 1]  (in place),  [X | y] = psi(q)^T S,  o = X / y' (y' = y if y > 0
 * else 1), i.e. o is the token's row of the full causal attention.  q (B,HQ,D), k (B,H,D),
 * v (B,H,Dv), o (B,HQ,Dv) of `dtype`; den (B,HQ) fp32 receives y (may be NULL).  `work` is
 * 16-byte aligned, of kata_decode_workspace_bytes(args) bytes; its first 4*B*HS bytes (tickets)
 * must be zero before the call and every call leaves them zero, so calls that share it run in
 * stream order, and a workspace reused for a larger B*HS is zeroed again first.  D <= 256.
 * ------------------------------------------------------------------------------------------- */
typedef struct {
  const void* q;
  const void* k;
  const void* v;
  const float* g;  /* (B,HQ) per-token log-decay, or NULL                 */
  float* state;    /* (B*HS, F, lds) fp32, updated in place              */
  void* o;
  float* den;      /* may be NULL                                        */
  void* work;
  int dtype, B, HQ, H, D, Dv, M, lds;
  int score;       /* KATA_SCORE_*                                       */
  float scale;
} kata_decode_args;

KATA_API size_t kata_decode_workspace_bytes(const kata_decode_args* args);
KATA_API int kata_decode_step(const kata_decode_args* args, kata_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Mixer prologue / epilogue (the operations kata/layer.py runs around the attention op).
 *
 * Causal depthwise short convolution with optional SiLU, as fla's ShortConvolution on q, k and v
 * (kata/layer.py:176-194 builds them, :305-319 applies them):
 *   y[b,t,c] = act(sum_{i<K} w[c*K + i] x[b, t-K+1+i, c] + bias[c]),  x = 0 before t = 0.
 * x rows are ldx elements apart (so q, k and v can be read as column ranges of one fused
 * projection output), y rows ldy apart, dx rows lddx apart; C, the strides and the pointers must
 * keep 16-byte alignment (C and strides multiples of 8 for 16-bit dtypes, of 4 for fp32).  Math in
 * fp32; w, bias, dw, dbias fp32; K <= 4.  Backward writes dx (dtype) and dw / dbias (fp32, written,
 * not accumulated) and needs kata_short_conv_bwd_workspace_bytes() of workspace; results do not
 * depend on scheduling (fixed-order reduction of per-CTA partials).
 * ------------------------------------------------------------------------------------------- */
typedef struct {
  const void* x;        /* (B, T, ldx) dtype: channels [0, C) of each row  */
  const float* w;       /* (C, K) fp32, nn.Conv1d's (C, 1, K) weight        */
  const float* bias;    /* (C) fp32 or NULL                                 */
  void* y;              /* forward: (B, T, ldy) dtype [out]                 */
  const void* dy;       /* backward: (B, T, ldy) dtype                      */
  void* dx;             /* backward: (B, T, lddx) dtype [out]               */
  float* dw;            /* backward: (C, K) fp32 [out]                      */
  float* dbias;         /* backward: (C) fp32 [out] or NULL                 */
  void* workspace;
  size_t workspace_bytes;
  int dtype;
  int B, T, C, K;
  long long ldx, ldy, lddx;
  int activation;       /* 0 none, 1 SiLU                                    */
} kata_conv_args;

KATA_API int kata_short_conv_fwd(const kata_conv_args* args, kata_stream_t stream);
KATA_API size_t kata_short_conv_bwd_workspace_bytes(const kata_conv_args* args);
KATA_API int kata_short_conv_bwd(const kata_conv_args* args, kata_stream_t stream);

/* Row normalisation with optional rotary embedding, over `rows` contiguous rows of N values (one
 * (token, head) slice each; row r is position (r / heads) % T):
 *   norm 1  l2:   y = x / sqrt(sum x^2 + eps)              (fla l2norm; kata/layer.py:346-347)
 *   norm 2  RMS:  y = x rsqrt(mean x^2 + eps) * w (w NULL: no scale)  (fla RMSNorm: the qk norm
 *                 of kata/layer.py:166-169 and the output norm over head_v_dim, :199-209, :539)
 *   norm 0  none
 * then, if rope != 0, the rotation of fla's RotaryEmbedding with tables cos/sin (T, R/2) fp32:
 *   rope 1  interleaved pairs (2f, 2f+1) over the whole row, R = N   (kata/layer.py:147-149)
 *   rope 2  inside every group of R values, value r < R/2 paired with r + R/2 (rope_group,
 *           kata/layer.py:139-141, :355-366); R/2 a multiple of 8 (16-bit) or 4 (fp32)
 * N/8 (16-bit) or N/4 (fp32) must be a power of two <= 32, or (normalisation only, rope 0) 64, 96, 128
 * or 192 (rows of up to 1536 16-bit values, e.g. a 768-wide hidden state).  Forward stores rstd (the per-row
 * 1/norm, fp32) when norm != 0; backward takes x, rstd, dy and writes dx, and dw (fp32, N) for RMS
 * with a weight, using kata_rownorm_bwd_workspace_bytes() of workspace.  No counterpart in the
 * reference as one operation: it fuses the separate fla kernels the layer calls.
 * ------------------------------------------------------------------------------------------- */
typedef struct {
  const void* x;        /* (rows, N) dtype                                   */
  const float* w;       /* (N) fp32 or NULL                                  */
  const float* cos;     /* (T, R/2) fp32 or NULL                             */
  const float* sin;     /* (T, R/2) fp32 or NULL                             */
  void* y;              /* forward: (rows, N) dtype [out]                    */
  float* rstd;          /* (rows) fp32: forward [out], backward [in]         */
  const void* dy;       /* backward: (rows, N) dtype                         */
  void* dx;             /* backward: (rows, N) dtype [out]                   */
  float* dw;            /* backward: (N) fp32 [out]                          */
  void* workspace;
  size_t workspace_bytes;
  int dtype;
  long long rows;
  int N, T, heads;
  int norm, rope, R;
  float eps;
} kata_rownorm_args;

KATA_API int kata_rownorm_fwd(const kata_rownorm_args* args, kata_stream_t stream);
KATA_API size_t kata_rownorm_bwd_workspace_bytes(const kata_rownorm_args* args);
KATA_API int kata_rownorm_bwd(const kata_rownorm_args* args, kata_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * The KATA LM's MLP activation and loss (kata/modeling.py's fla GatedMLP with fuse_swiglu and the
 * fused cross entropy of LinearAttentionForCausalLM), for the config-5 training step.
 *   SwiGLU: gu is (rows, 2I) = [g | u] (the fused gate/up projection), y = silu(g) u (rows, I);
 *   backward writes dgu = [dy u silu'(g) | dy silu(g)].  I a multiple of 8 (16-bit) or 4 (fp32).
 *   Cross entropy over rows of V logits with int64 targets (target < 0: ignored row):
 *   forward writes lse (rows, fp32) and loss_rows = lse - logit[target] (0 when ignored);
 *   backward writes dlogits = (softmax - onehot) * grad_loss[0] * inv_count[0] (0 for ignored rows),
 *   both scalars read on the device.  One read of the logits forward, one read and one write
 *   backward; no fp32 copy of the logits.  No counterpart in the reference's own code (fla kernels).
 * ------------------------------------------------------------------------------------------- */
KATA_API int kata_swiglu_fwd(const void* gu, void* y, long long rows, int I, int dtype, kata_stream_t stream);
KATA_API int kata_swiglu_bwd(const void* gu, const void* dy, void* dgu, long long rows, int I, int dtype,
                             kata_stream_t stream);
KATA_API int kata_cross_entropy_fwd(const void* logits, const int64_t* targets, float* lse, float* loss_rows,
                                    long long rows, int V, int dtype, kata_stream_t stream);
KATA_API int kata_cross_entropy_bwd(const void* logits, const int64_t* targets, const float* lse,
                                    const float* grad_loss, const float* inv_count, void* dlogits, long long rows,
                                    int V, int dtype, kata_stream_t stream);

/* Residual add + RMSNorm of the LM's hidden stream (fla's fused add-norm between the blocks of the
 * reference model, kata/modeling.py): forward h_out = h + x (fp32), y = h_out rsqrt(mean h_out^2 + eps) w
 * in x's dtype (bf16 / f16), rstd per row; backward dh = dh_in + d(RMSNorm)/dh_out (fp32; dh_in may be
 * NULL), dx = dh in x's dtype (either output may be NULL), dw (fp32, reduced in a fixed order over
 * kata_add_rmsnorm_bwd_workspace_bytes() of partials).  Rows of N values, N a multiple of 256 up to
 * 1024; every pointer 16-byte aligned. */
typedef struct {
  const float* h;      /* (rows, N) fp32 residual stream          [fwd in]  */
  const void* x;       /* (rows, N) dtype, the block output       [fwd in]  */
  const float* w;      /* (N) fp32 norm weight                    [in]      */
  float* h_out;        /* (rows, N) fp32 h + x    [fwd out; bwd in]         */
  void* y;             /* (rows, N) dtype normalised              [fwd out] */
  float* rstd;         /* (rows) fp32             [fwd out; bwd in]         */
  const void* dy;      /* (rows, N) dtype                         [bwd in]  */
  const float* dh_in;  /* (rows, N) fp32 gradient of h_out's other uses, or NULL [bwd in] */
  float* dh;           /* (rows, N) fp32                          [bwd out] */
  void* dx;            /* (rows, N) dtype                         [bwd out] */
  float* dw;           /* (N) fp32                                [bwd out] */
  void* workspace;
  size_t workspace_bytes;
  long long rows;
  int N;
  int dtype;
  float eps;
} kata_add_rmsnorm_args;

KATA_API int kata_add_rmsnorm_fwd(const kata_add_rmsnorm_args* args, kata_stream_t stream);
KATA_API size_t kata_add_rmsnorm_bwd_workspace_bytes(const kata_add_rmsnorm_args* args);
KATA_API int kata_add_rmsnorm_bwd(const kata_add_rmsnorm_args* args, kata_stream_t stream);

/* Human-readable name of a KATA_ERR_* code (static storage). */
KATA_API const char* kata_strerror(int code);

/* ABI revision of this header; bumped on any incompatible change. */
KATA_API int kata_abi_version(void);
#define KATA_ABI_VERSION 2

/* Diagnostic: D(M x N, fp32, row-major) = A * B^T through one CTA of TMA loads and tcgen05 MMAs.
 * A is (M x K) bf16, stored K-contiguous when a_mn == 0 or as (K x M) M-contiguous when a_mn == 1;
 * B is (N x K) K-contiguous when b_mn == 0 or (K x N) N-contiguous when b_mn == 1.  *_sw is the
 * shared-memory swizzle span in bytes (32, 64 or 128).  a_tmem == 1 stages A in tensor memory
 * (tcgen05.st) instead of shared memory.  M == 128; N, K multiples of 16, <= 256.
 * No counterpart in the reference: it checks this library's descriptor encodings on the device. */
KATA_API int kata_selftest_umma(const void* A, const void* B, float* D, int M, int N, int K, int a_mn, int b_mn,
                       int a_sw, int b_sw, int a_tmem, kata_stream_t stream);

/* Diagnostic: the same with M == 64 (the 64-token chunk tiles of the gated delta rule), both operands
 * in 128-byte swizzled shared memory, and the accumulator at TMEM lane offset lane_off (0 or 16):
 * checks that row m of an M = 64 accumulator sits in lane (m % 16) + 32 * (m / 16) + lane_off.
 * No counterpart in the reference. */
KATA_API int kata_selftest_umma_m64(const void* A, const void* B, float* D, int N, int K, int a_mn, int b_mn,
                                    int lane_off, kata_stream_t stream);

/* Diagnostic: D (256 x N, fp32) = A * B^T through one CTA pair (a cluster of two CTAs running
 * cta_group::2 MMAs with M = 256).  Each CTA loads its 128 rows of A and its half of B (N/2 rows of a
 * K-contiguous B, N/2 columns of an N-contiguous one); a_tmem == 1 stages A in tensor memory (only
 * with a_mn == 0).  N a multiple of 32 in [32, 256]; K a multiple of 16, <= 256.
 * No counterpart in the reference: it checks the pair layout used by the attention kernels. */
KATA_API int kata_selftest_umma_pair(const void* A, const void* B, float* D, int N, int K, int a_mn, int b_mn,
                                     int a_sw, int b_sw, int a_tmem, kata_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* KATA_B200_H */
