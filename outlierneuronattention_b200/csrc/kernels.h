// Internal launch interface between the C ABI (capi.cu) and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace hofa {

struct DecodeParams {
  const void* q; const void* k; const void* v;
  const void* cache_k; const void* cache_v;
  const float* state_in; float* state_out;
  const void* log_gamma; const void* mix_g; const void* norm_w; const void* log_alpha;
  void* y;
  int B, H, D, R;
  int L;                      // cache capacity (rows)
  int seq_len;
  const int* seq_len_dev;
  float qk_scale_log2;        // sm_scale * log2(e)
  float eps;
  int split_k;
  int64_t sq[3], sk[3], sv[3];  // b, h, d
  int64_t sck[4], scv[4];       // b, h, t, d
  int64_t sst[3], sso[3];       // b, h, row  (d stride is 1)
  int64_t slg[2], smg[2];       // b, h
  int64_t snw[2];               // h, d
  int64_t sla[3];               // b, h, j
  int64_t sy[3];                // b, h, d
  int dt_lg, dt_mg, dt_nw, dt_la;
  float* ws_part;
  int* ws_count;
  int* ws_status;
  int stages;                 // bulk ring depth (64-token chunks)
  int consumer_warps;         // bulk kernel consumer warps: 4, 6 or 8
  bool no_l2_prefetch;        // bulk kernel: skip the L2 prefetch of the cache rows before the grid dependency
  bool prefetch_window;       // bulk kernel: that prefetch covers only the ring's first window of chunks
  // hofa_decode_step_fwd (bulk kernel): the new token's gates, RoPE and cache
  // row are computed in the same launch.  q, k, v are then un-rotated; the
  // cache is streamed over rows [0, seq_len - 1) and the new token (row
  // seq_len - 1) joins the softmax from registers; log_gamma / mix_g above
  // are unused (log_gamma_out / mix_out, when non-null, receive them).
  bool fused_prep;
  const void* gate_w; const void* gate_b; const void* mix_w; const void* mix_b; const void* fixed_mix;
  const void* rope_cos; const void* rope_sin;
  void* log_gamma_out; void* mix_out;
  int rope_rows;              // rows of the RoPE tables (0: no RoPE)
  int64_t sgw[2], sgb, smw[2], smb, sfm, scos[2], ssin[2], slgo[2], smo[2];
  int dt_gw, dt_gb, dt_mw, dt_mb, dt_fm, dt_cs, dt_lgo, dt_mo;
};

// path: 0 = strided register loads, 1 = 16-byte register loads, 2 = TMA bulk ring
cudaError_t launch_decode(const DecodeParams& p, int dtype, int path, bool alpha, cudaStream_t st);

struct GlaParams {
  const void* q; const void* k; const void* v;
  const void* log_gamma; const void* log_alpha; const void* mix_g; const void* gla_scale;
  const float* state_init;
  void* y;
  float* state_out;
  int B, H, T, D, R, J;
  int chunk;
  int nseg;                   // segments per (b,h)
  int seg_len;                // tokens per segment (multiple of chunk)
  float eps;
  bool fuse;                  // mix_g and gla_scale present
  int64_t sq[4], sk[4], sv[4], sy[4];
  int64_t slg[3], smg[3];
  int64_t sla[3];
  int64_t sgs[2];
  int64_t ssi[3], sso[4];     // state_init b,h,row ; state_out b,h,row,d
  int dt_lg, dt_mg, dt_la, dt_gs;
  float* ws_state;            // [B,H,nseg,J,D] local end states
  float* ws_decay;            // [B,H,nseg,J] log of the segment's total decay
  // single-launch tensor-core form (head dim 64): chunk tickets, per-chunk
  // publication flags, each chunk's state contribution and the state after it
  unsigned* ws_ticket;
  unsigned long long* ws_flags;  // [B*H*nseg]: state in the low word, the chunk's log decay (f32 bits) in the high
  float* ws_agg;              // [B*H*nseg, J, D]
  float* ws_incl;             // [B*H*nseg, J, D]
};

cudaError_t launch_gla(const GlaParams& p, int dtype, cudaStream_t st);

struct OutlierParams {
  const void* q; const void* k; const void* v; const void* mix_g;
  void* out;
  int B, H, Tq, Tk, D, R;
  int q_offset;
  float qk_scale_log2;
  bool accumulate;
  int64_t sq[4], sk[4], sv[4], so[4];
  int64_t smg[3];
  int dt_mg;
};

cudaError_t launch_outlier(const OutlierParams& p, int dtype, cudaStream_t st);

struct PrepParams {
  void* q; void* k; const void* v;
  const void* gate_w; const void* gate_b;
  const void* mix_w; const void* mix_b; const void* fixed_mix;
  const void* cos; const void* sin;
  void* log_gamma; void* mix_out;
  void* cache_k; void* cache_v;
  int B, H, N, D, R;
  int pos0; const int* pos0_dev;
  int pos0_dev_bias;           // added to *pos0_dev (a device seq_len gives position seq_len - 1)
  int L;                       // cache rows (bound for the append)
  int P;                       // rows of the RoPE tables
  bool rope;
  int64_t sq[4], sk[4], sv[4];
  int64_t sgw[2], sgb, smw[2], smb, sfm;
  int64_t scos[2], ssin[2];
  int64_t slg[3], smo[3];
  int64_t sck[4], scv[4];
  int dt_gw, dt_gb, dt_mw, dt_mb, dt_fm, dt_cs, dt_lg, dt_mo;
  bool vec;                    // unit channel strides and 16-byte aligned rows everywhere
  uint32_t zero;               // 0, set by the launcher (an operand the compiler cannot fold)
};

cudaError_t launch_prep(const PrepParams& p, int dtype, cudaStream_t st);

}  // namespace hofa
