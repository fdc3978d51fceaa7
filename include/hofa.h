/*
 * hofa.h -- C ABI of the B200-native HOFA attention hot path (libhofa_b200.so).
 *
 * HOFA = Hybrid Outlier-Factorized Attention (LotanGutman/OutlierNeuronAttention).
 * Each head's q/k channels are split: channels [0, R) go to exact causal
 * softmax attention ("outlier" path, full-width V), channels [R, D) to a gated
 * linear attention recurrence ("inlier" path, GLA).  A per-token sigmoid gate
 * mix blends them: Y = mix * Y_O + (1 - mix) * gla_scale * RMSNorm(Y_I).
 *
 * Every entry point below replaces one operator of the reference (cited per
 * function as file:line of the reference checkout).  The signatures carry
 * plain device pointers, element strides, shapes, dtype codes and scalars; no
 * framework types cross this boundary.  All launches are asynchronous on the
 * given cudaStream_t (passed as void*), never synchronise, never allocate, and
 * can be captured in a CUDA graph.  A non-zero return is a hofa_status; the
 * message of the last failure on the calling thread is hofa_last_error().
 */
#ifndef HOFA_B200_H
#define HOFA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HOFA_ABI_VERSION 1

typedef enum hofa_status {
  HOFA_OK = 0,
  HOFA_ERR_INVALID_ARGUMENT = 1, /* shape, stride, dtype or scalar out of contract */
  HOFA_ERR_UNSUPPORTED = 2,      /* valid for the reference, not built here (e.g. head dim 96) */
  HOFA_ERR_MISALIGNED = 3,       /* a pointer the kernel streams is not 16-byte aligned */
  HOFA_ERR_WORKSPACE = 4,        /* workspace missing or smaller than *_workspace_size() */
  HOFA_ERR_CUDA = 5              /* a CUDA runtime call failed (launch error) */
} hofa_status;

typedef enum hofa_dtype {
  HOFA_DTYPE_F32 = 0,
  HOFA_DTYPE_BF16 = 1,
  HOFA_DTYPE_F16 = 2
} hofa_dtype;

/* A strided view of device memory.  data == NULL marks an absent optional
 * tensor.  shape/stride are in elements, outermost first; unused trailing
 * dims have shape 1. */
typedef struct hofa_tensor {
  void* data;
  int32_t dtype;   /* hofa_dtype */
  int32_t ndim;    /* 1..4 */
  int64_t shape[4];
  int64_t stride[4];
} hofa_tensor;

/* ------------------------------------------------------------------------ */
/* Decode: one token of the attention core.                                  */
/* ------------------------------------------------------------------------ */
typedef struct hofa_decode_args {
  hofa_tensor q, k, v;     /* [B,H,1,D]; q[..., :R] RoPE-rotated, k/v of the new token */
  hofa_tensor cache_k;     /* [B,H,L,>=R] rotated outlier keys; rows [0, seq_len) are read */
  hofa_tensor cache_v;     /* [B,H,L,D] values */
  hofa_tensor state_in;    /* [B,H,D-R,D] f32 GLA state (read) */
  hofa_tensor state_out;   /* [B,H,D-R,D] f32 GLA state (written); may not alias state_in */
  hofa_tensor log_gamma;   /* [B,H,1] log decay of this token */
  hofa_tensor mix_g;       /* [B,H,1] blend gate in [0,1] */
  hofa_tensor norm_w;      /* [H,D] gla_scale */
  hofa_tensor log_alpha;   /* optional [1|B,H,1,D-R] per-channel decay exponent (log) */
  hofa_tensor y;           /* [B,H,1,D] output, dtype of q */
  int32_t R;               /* outlier channels, 0..D (R == 0: no outlier term, y = gla_scale*RMSNorm(y_I)
                              when mix_g is 0 -- the layer's r = 0 decode) */
  int32_t seq_len;         /* cache rows to attend; used when seq_len_dev == NULL */
  const int32_t* seq_len_dev; /* optional device int32 read at run time (CUDA-graph replay
                                 with an advancing position); values outside [1, L] are
                                 clamped and flagged in the workspace status word */
  float sm_scale;          /* logit scale, sqrt(D/R) in the layer */
  float eps;               /* RMSNorm epsilon (reference decode: FLT_EPSILON) */
  int32_t split_k;         /* cache splits per (b,h); 0 = choose automatically */
  void* workspace;         /* >= hofa_decode_workspace_size(B,H,D,split_k) bytes, zero-filled
                              once after allocation; every launch leaves it reusable */
  size_t workspace_bytes;
} hofa_decode_args;

/* Replaces fused_hofa_decode (src/hofa_decode_triton.py:342-476) and its three
 * Triton kernels (:47-159 single pass, :172-239 split, :241-340 reduce) with
 * ONE launch: split-K streaming of the cache, GLA update/readout distributed
 * over the splits, last-CTA combine, RMSNorm and blend. */
int hofa_decode_fwd(const hofa_decode_args* args, void* stream);

/* Workspace bytes for hofa_decode_fwd with at most max_split_k splits
 * (max_split_k <= 0: the largest split the automatic choice can make). */
size_t hofa_decode_workspace_size(int32_t B, int32_t H, int32_t D, int32_t max_split_k);

/* The automatic split count for (B, H, seq_len) on a GPU with num_sms SMs;
 * replaces the heuristic at src/hofa_decode_triton.py:374-383. */
int32_t hofa_decode_choose_split(int32_t B, int32_t H, int32_t seq_len, int32_t num_sms);

/* Status word the decode kernel leaves in its workspace, then clears it.
 * 0 = no fault; bits: 1 = seq_len_dev held a value outside [1, L] and was
 * clamped; 4 / 8 = a ring wait of the TMA-bulk kernel timed out (producer /
 * consumer); 16 = invalid ring configuration; 64 = the cluster combine's wait
 * for the other splits timed out.
 * Synchronises `stream`; not for use inside graph capture. */
int hofa_decode_read_status(void* workspace, void* stream, int32_t* status_out);

/* Same decode step as hofa_decode_fwd for callers that cannot allocate
 * device memory (a host runtime that owns all allocations, a real-time loop
 * that must not enter the driver's allocator, glue holding only borrowed
 * pointers).  No counterpart in the reference.  args->workspace and
 * args->workspace_bytes are ignored: the scratch is a 2 MiB array built into
 * the library (held on every GPU that loads it until exit), and calls needing
 * more (hofa_decode_workspace_size of their B, H, D and split count) fail with
 * HOFA_ERR_WORKSPACE.  All arguments are validated, and the split count
 * chosen, exactly as hofa_decode_fwd does before anything is issued.  All
 * calls share that array, so calls that overlap on the GPU race and must be
 * serialised by the caller.  The first call on a device looks up the array's
 * address; make it before any stream capture.  Each call clears the array's
 * combine tickets on `stream` before the kernel; the status word keeps the
 * bits of every call until hofa_decode_noalloc_read_status reads it.  It never
 * allocates. */
int hofa_decode_fwd_noalloc(const hofa_decode_args* args, void* stream);

/* The status word of hofa_decode_fwd_noalloc's built-in scratch on the current
 * device (the bits of hofa_decode_read_status, collected over every call since
 * the last read), then clears it.  No counterpart in the reference.
 * Synchronises `stream`; not for use inside graph capture. */
int hofa_decode_noalloc_read_status(void* stream, int32_t* status_out);

/* ------------------------------------------------------------------------ */
/* Prefill, inlier path: chunked gated linear attention.                      */
/* ------------------------------------------------------------------------ */
typedef struct hofa_gla_args {
  hofa_tensor q, k, v;     /* [B,H,T,D]; inlier channels are q/k[..., R:D] */
  hofa_tensor log_gamma;   /* [B,H,T] */
  hofa_tensor log_alpha;   /* optional [1|B,H,1,D-R] */
  hofa_tensor mix_g;       /* optional [B,H,T]; with gla_scale enables the fused epilogue */
  hofa_tensor gla_scale;   /* optional [H,D] */
  hofa_tensor state_init;  /* optional [B,H,D-R,D] f32 state before token 0 (zero if absent) */
  hofa_tensor y;           /* [B,H,T,D] out: (1-mix)*gla_scale*RMSNorm(y_I), or raw y_I */
  hofa_tensor state_out;   /* optional [B,H,D-R,D] f32 final state */
  int32_t R;
  int32_t chunk_size;      /* tokens per chunk (reference default 64); 16..64, multiple of 16 */
  float eps;               /* RMSNorm epsilon (reference operator: 1e-5) */
  int32_t num_segments;    /* sequence segments per (b,h) run in parallel; 0 = automatic */
  void* workspace;         /* >= hofa_gla_workspace_size(...) bytes (no initialisation needed) */
  size_t workspace_bytes;
} hofa_gla_args;

/* Replaces chunk_gla_inlier_fwd (src/chunk_gla_inlier.py:153-237) and
 * chunk_gla_fwd_kernel (:5-150).  bf16/f16 inputs with R % 8 == 0 run
 * chunk-parallel tcgen05 kernels when the workspace holds
 * hofa_gla_workspace_size() bytes: at D = 64 with a scalar decay one launch
 * (the state carried between chunks by a look-back inside the launch; the
 * call also clears the front of the workspace, so it needs no
 * initialisation), otherwise three (per-chunk state contributions, a scan
 * over chunks, per-chunk outputs), a per-channel decay (log_alpha) included.
 * Other cases run a segment-parallel CUDA-core kernel.  Calls that share a
 * workspace must not run concurrently. */
int hofa_prefill_gla_fwd(const hofa_gla_args* args, void* stream);
size_t hofa_gla_workspace_size(int32_t B, int32_t H, int32_t T, int32_t D, int32_t R,
                               int32_t chunk_size, int32_t num_segments);

/* ------------------------------------------------------------------------ */
/* Prefill, outlier path: causal softmax attention on R channels.            */
/* ------------------------------------------------------------------------ */
typedef struct hofa_outlier_args {
  hofa_tensor q;           /* [B,H,Tq,>=R]; channels [0,R) used, RoPE-rotated */
  hofa_tensor k;           /* [B,H,Tk,>=R] */
  hofa_tensor v;           /* [B,H,Tk,D] */
  hofa_tensor mix_g;       /* [B,H,Tq] */
  hofa_tensor out;         /* [B,H,Tq,D] in/out */
  int32_t R;
  int32_t q_offset;        /* key j is visible to query i iff j <= i + q_offset (reference: 0) */
  float sm_scale;          /* sqrt(D/R) in the layer */
  int32_t accumulate;      /* 1: out += mix*attn (reference semantics); 0: out = mix*attn */
} hofa_outlier_args;

/* Replaces exact_attention_triton (src/exact_attention.py:163-188) and its
 * kernel _fwd_kernel (:45-161).  bf16/f16 inputs with D in {64, 128} and
 * R in {16, 32, 64} run on the tcgen05 tensor-core kernel (TMA-fed, TMEM
 * accumulators); other shapes and float32 inputs on a CUDA-core kernel. */
int hofa_prefill_outlier_fwd(const hofa_outlier_args* args, void* stream);

/* Device status of the tensor-core prefill kernels since the last read (0 = no
 * fault; bit 0: outlier attention, bit 1: GLA -- a bounded wait for a copy or
 * an MMA ran out and the affected rows were not written), then clears it.
 * Synchronises `stream`. */
int hofa_prefill_read_status(void* stream, int32_t* status_out);

/* ------------------------------------------------------------------------ */
/* Gates + RoPE + cache export (prefill and decode step).                     */
/* ------------------------------------------------------------------------ */
typedef struct hofa_prep_args {
  hofa_tensor q, k;        /* [B,H,N,D] un-rotated projections; channels [0,R) are RoPE-rotated IN PLACE */
  hofa_tensor v;           /* [B,H,N,D] (read only when cache_v is given) */
  hofa_tensor gate_w;      /* [H,2D] gate_proj.weight (first D columns act on q) */
  hofa_tensor gate_b;      /* [H] */
  hofa_tensor mix_w;       /* optional [H,2D] mix_proj.weight */
  hofa_tensor mix_b;       /* optional [H] */
  hofa_tensor fixed_mix;   /* optional [H] fixed_mix logits (fixed_blend_weight ablation) */
  hofa_tensor cos, sin;    /* [P,R] RoPE tables (RotaryEmbedding.cos_cached / sin_cached) */
  hofa_tensor log_gamma;   /* out [B,H,N]: logsigmoid(-gate) */
  hofa_tensor mix_out;     /* optional out [B,H,N]: sigmoid(mix logits) */
  hofa_tensor cache_k;     /* optional out [B,H,L,>=R]: rows pos0..pos0+N-1 get the rotated k */
  hofa_tensor cache_v;     /* optional out [B,H,L,D]: same rows get v */
  int32_t R;               /* rotated channels (0: gates only) */
  int32_t pos0;            /* absolute position of token 0; used when pos0_dev == NULL */
  const int32_t* pos0_dev; /* optional device int32 */
  int32_t use_rope;
} hofa_prep_args;

/* Replaces the module-side glue of the layer: _compute_gates_optimized
 * (src/HybridOutlierFactorizedAttention.py:67-95), logsigmoid (:177, :361),
 * RoPE (:180-188, :365-375; src/modules/modules.py:33-45) and the cache
 * export / append (:196-198, :382-384). */
int hofa_prep_fwd(const hofa_prep_args* args, void* stream);

/* One decode step of the layer with the new token's prep fused in: the same
 * result as hofa_prep_fwd(prep) followed by hofa_decode_fwd(decode) with
 * decode.log_gamma = prep.log_gamma and decode.mix_g = prep.mix_out, where the
 * new token's position is decode.seq_len - 1 (*decode.seq_len_dev - 1 when
 * that is given; prep.pos0 / pos0_dev are ignored).  prep.q/k/v must be
 * decode.q/k/v (one un-rotated token), prep.cache_k/v decode.cache_k/v, and
 * prep.mix_out is required.  On the TMA-bulk decode path this is one launch:
 * the cache is streamed over rows [0, seq_len - 1) while the new row, written
 * by the same launch, joins the softmax from registers; other paths run the
 * two launches.  The contents of q and k afterwards are unspecified (the
 * two-launch form rotates them in place, the fused form leaves them).
 * Replaces the layer's decode sequence at
 * src/HybridOutlierFactorizedAttention.py:360-416 (gates, RoPE at p, cache
 * append, fused_hofa_decode). */
int hofa_decode_step_fwd(const hofa_decode_args* decode, const hofa_prep_args* prep, void* stream);

/* ------------------------------------------------------------------------ */
/* Decoder-LM harness: small-batch linear layer (decode steps).               */
/* ------------------------------------------------------------------------ */
typedef struct hofa_linear_args {
  hofa_tensor x;           /* [M, K] input rows (M <= 8), or [M, 2K] = [gate | up] with input_mode 2 */
  hofa_tensor weight;      /* [N, K] (nn.Linear layout), K % 8 == 0, K <= 4096 */
  hofa_tensor norm_w;      /* [K] RMSNorm weight (input_mode 1) */
  hofa_tensor residual;    /* optional [M, N], added to the product; may be y itself */
  hofa_tensor y;           /* [M, N] output */
  int32_t input_mode;      /* 0: x; 1: RMSNorm(x) * norm_w; 2: silu(gate) * up */
  float eps;               /* RMSNorm epsilon */
} hofa_linear_args;

/* y = (residual +) transform(x) W^T for decode-sized batches, bf16 or f16:
 * the projections and MLP of the decoder LM that surrounds the HOFA layer in
 * the full-model decode benchmark (a SwiGLU / RMSNorm LM; the reference's own
 * LM wrappers, src/HybridOutlierFactorizedAttention.py:425-513, run them as
 * separate nn.Linear / LayerNorm / activation launches).  No counterpart
 * operator in the reference.  The input transform (RMSNorm or the SwiGLU
 * product, rounded to the activation dtype) and the residual add are fused
 * into the weight-streaming kernel.  Launched as a programmatic dependent
 * launch whose weight fetch starts before the previous kernel on the stream
 * has finished: the weight and norm_w must not be written by the kernel
 * immediately before this call on the stream (x and residual may be). */
int hofa_lm_linear_fwd(const hofa_linear_args* args, void* stream);

/* ------------------------------------------------------------------------ */
const char* hofa_last_error(void);
int32_t hofa_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* HOFA_B200_H */
