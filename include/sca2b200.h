/*
 * sca2b200 -- C ABI of the B200 (sm_100a) decayed-state / delta-rule scan.
 *
 * One recurrence covers every C-head / long-head variant of the reference
 * (per batch b, head h; fp32 state S in R^{K x V}):
 *
 *     S~_t = diag(gamma_t) S_{t-1}          gamma_t[m] = exp(g_t) * exp(-lam[m])
 *     e_t  = v_t - beta_t * (k_t^T S~_t) / kappa
 *     S_t  = S~_t + k_t e_t^T
 *     o_t  = Q_t^T S_t / kappa              (R read columns)
 *
 * Two input flavours:
 *   SCA2_FLAVOR_PHASE  phase-coded heads.  Inputs are the write phase phi and the
 *                      read phase psi (fp32, Mh modes); k = [cos phi ; sin phi]
 *                      (K = 2 Mh), kappa = Mh, R = 2 with the read columns
 *                      c1 = wr cos psi + wi sin psi, c2 = wr sin psi - wi cos psi:
 *                      o_re = c1.sr + c2.si, o_im = c1.si - c2.sr.
 *                      Replaces the chunk loop of LongHead._batched / _chunk
 *                      (lapa/layer.py:241-366), CHeadDeltaDamp._prefill_batched
 *                      (sca2/arch_damp.py:141-198), CHeadDelta._prefill_chunk
 *                      (sca2/arch_cdelta.py:137-172) and CHeadGated._chunk
 *                      (sca2/arch_gatedc.py:121-169).
 *   SCA2_FLAVOR_KEY    explicit keys (GDN form).  k, q given (K channels), R = 1,
 *                      kappa = 1, Q = q_scale * q; with v_times_beta = 1 the value
 *                      is pre-scaled by beta (write-gated GDN, e = beta (v - k^T S~)).
 *                      Replaces fla's naive_chunk_gated_delta_rule as called at
 *                      lapa/benchmarks/baselines.py:111-120.
 *
 * Conventions
 *   - All pointers are device pointers on the current device; all launches go
 *     on the given stream; no call synchronises the host or allocates memory.
 *   - Per-token tensors are passed as {ptr, stride_b, stride_t, stride_h} in
 *     ELEMENTS; the innermost (channel) dimension is contiguous.
 *   - Outputs o and dO carry a fourth stride, over the read column r.
 *   - State tensors are dense (B, H, K, V) fp32; for the phase flavour rows
 *     [0, Mh) hold the real part sr and rows [Mh, 2Mh) the imaginary part si.
 *   - Optional inputs (beta, g, lam, S0, dS_final) may be NULL; NULL beta is
 *     the additive write, NULL g / lam mean no decay of that kind.
 *   - lam * chunk must stay below ~80 (the closed form forms exp(+lam i) in
 *     fp32; the reference's guard is lam * chunk < 60, lapa/layer.py:39-43).
 *   - Return value: SCA2_OK, or an error code; sca2_last_error() gives the
 *     message (thread-local).  Invalid arguments are rejected on the host
 *     before any launch.
 */
#ifndef SCA2B200_H
#define SCA2B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SCA2_API __attribute__((visibility("default")))
#else
#define SCA2_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum sca2_status {
  SCA2_OK = 0,
  SCA2_ERR_ARG = 1,       /* invalid argument (shape, stride, null, dtype) */
  SCA2_ERR_UNSUPPORTED = 2,
  SCA2_ERR_CUDA = 3,      /* a CUDA runtime call or launch failed */
};

enum sca2_dtype { SCA2_F32 = 0, SCA2_BF16 = 1 };
enum sca2_flavor { SCA2_FLAVOR_PHASE = 0, SCA2_FLAVOR_KEY = 1 };

/* One per-token tensor: element (b, t, h, c) at ptr[b*sb + t*st + h*sh + c]. */
typedef struct sca2_tok {
  const void* ptr;
  int64_t sb, st, sh;
} sca2_tok;

/* Output per-token tensor with a read-column stride: (b,t,h,r,c). */
typedef struct sca2_out {
  void* ptr;
  int64_t sb, st, sh, sr;
} sca2_out;

typedef struct sca2_scan_args {
  int32_t flavor;       /* sca2_flavor */
  int32_t B, T, H;
  int32_t K;            /* key width: 2*Mh (phase) or K (key flavour) */
  int32_t V;            /* value width */
  int32_t io_dtype;     /* dtype of v, q, k (key flavour), o, dO, dv */
  int32_t v_times_beta; /* key flavour: value pre-scaled by beta (GDN) */
  float q_scale;        /* key flavour: Q = q_scale * q */
  /* inputs */
  sca2_tok phw;         /* phase: write phase phi (fp32, Mh)   | key: k (io dtype, K) */
  sca2_tok phq;         /* phase: read phase psi (fp32, Mh)    | key: q (io dtype, K) */
  sca2_tok v;           /* value (io dtype, V) */
  sca2_tok beta;        /* erase gate, fp32, one channel; ptr NULL = additive */
  sca2_tok g;           /* scalar log-decay <= 0, fp32; ptr NULL = none */
  const float* lam;     /* (H, Mh) phase / (H, K) key, >= 0; NULL = none */
  const float* wr;      /* (H, Mh) phase only */
  const float* wi;      /* (H, Mh) phase only */
  const float* S0;      /* (B,H,K,V) incoming state; NULL = zeros */
} sca2_scan_args;

/* Forward scan.
 *   o             (b,t,h,r,V) raw read, io dtype (R = 2 phase, 1 key)
 *   S_final       (B,H,K,V) fp32 or NULL
 *   chunk_states  NULL, or (B,H,NC,K,V) fp32 with NC = sca2_num_chunks(T): the
 *                 state entering every chunk, kept for the backward.
 * Replaces the forward of the reference's prefill paths listed above. */
SCA2_API int sca2_scan_fwd(const sca2_scan_args* a, sca2_out o, float* S_final,
                  float* chunk_states, void* stream);

/* 1 if a training forward (sca2_scan_fwd with a 16-byte aligned chunk_states buffer) of these
 * arguments runs the chunk-parallel kernels with the value tile of every full 64-token chunk
 * loaded by one TMA tensor copy (phase flavour, bf16 values, K = V = 64, few sequences,
 * T % 8 == 0, 16-byte aligned value rows with the batches contiguous), else 0.  A diagnostic:
 * no counterpart in the reference. */
SCA2_API int sca2_scan_value_tma(const sca2_scan_args* a);

/* Number of slots of the saved-state buffer for T tokens (four per 64-token chunk: the
 * state entering the chunk, and the chunk's saved intermediates for the backward). */
SCA2_API int32_t sca2_num_chunks(int32_t T);

/* Gradients written by sca2_scan_bwd.  All per-token gradient buffers except dv
 * are fp32 and ACCUMULATED INTO (the caller zero-fills them); dv is written in the
 * io dtype.  Per-head gradients (dlam, dwr, dwi) are fp32 and accumulated into.
 *   dphw / dphq : phase: d phi, d psi (Mh)     | key: dk, dq (K)
 *   dv          : (io dtype, V)
 *   dbeta, dg   : one channel, fp32 (ignored where the input was NULL)
 *   dlam        : (H, Mh) phase / (H, K) key, or NULL
 *   dwr, dwi    : (H, Mh) phase, or NULL
 *   dS0         : (B,H,K,V) fp32 gradient of the incoming state (written), or NULL
 */
typedef struct sca2_scan_grads {
  sca2_tok dphw, dphq, dv, dbeta, dg;
  float* dlam;
  float* dwr;
  float* dwi;
  float* dS0;
  /* 0: the fp32 gradients are accumulated into (caller zero-fills them, as above).
   * 1: every gradient is WRITTEN: the library initialises the buffers itself (the
   *    tensor-core backward writes the per-token rows directly where one CTA owns them)
   *    and all per-token gradient tensors must be dense (B,T,H,C). */
  int32_t overwrite;
  /* 0: dk / dq (key flavour) are fp32.  1: they are written in the io dtype, like dv (key
   * flavour, overwrite mode; supported where the chunk-parallel path runs: bf16, K = V = 128,
   * no lam, 16-byte aligned rows); elsewhere the call fails with SCA2_ERR_UNSUPPORTED. */
  int32_t grad_io_dtype;
} sca2_scan_grads;

/* Backward scan: reverse chunk sweep of the adjoint state, all per-token
 * gradients of a chunk from (state entering the chunk, adjoint leaving it).
 *   dO            (b,t,h,r,V) io dtype, upstream gradient of o
 *   dS_final      (B,H,K,V) fp32 upstream gradient of S_final, or NULL
 *   chunk_states  as written by sca2_scan_fwd for the same inputs.  The explicit-key path at
 *                 K = V = 128 also uses its free parts as the backward's workspace (the
 *                 forward's saved data stay intact, so the backward may be repeated).
 * Replaces torch autograd through the reference's prefill (sca2/arch_damp.py:141-198,
 * lapa/layer.py:298-366). */
SCA2_API int sca2_scan_bwd(const sca2_scan_args* a, sca2_out dO, const float* dS_final,
                  float* chunk_states, const sca2_scan_grads* gr, void* stream);

/* Single-token decode step for every (b, h): read S (B,H,K,V) fp32, write the new
 * state to S_out (may equal S_in) and the read o (b,h,r,V).  Per-token inputs use
 * sca2_tok with T = 1 (st ignored).  Replaces LongHead.step (lapa/layer.py:387-412),
 * CHeadDeltaDamp.step (sca2/arch_damp.py:225-245), CHeadDelta.step
 * (sca2/arch_cdelta.py:186-206), CHeadGated.step (sca2/arch_gatedc.py:171-193) and
 * fla's naive_recurrent_gated_delta_rule with T = 1 (lapa/benchmarks/baselines.py:142). */
SCA2_API int sca2_scan_step(const sca2_scan_args* a, const float* S_in, float* S_out,
                   sca2_out o, void* stream);

/* Per-row RMS read-out u = x * rsqrt(mean(x^2) + eps) over the last dim D, with
 * x (N, D) io dtype contiguous rows and u in the same dtype (sca2/ref.py:29-30,
 * lapa/layer.py:117-118). */
SCA2_API int sca2_rms_fwd(const void* x, void* u, int64_t N, int32_t D, float eps,
                 int32_t io_dtype, void* stream);
/* dx = (du - u * mean(du * u)) * rsqrt(mean(x^2) + eps); dx may alias du. */
SCA2_API int sca2_rms_bwd(const void* x, const void* du, void* dx, int64_t N, int32_t D,
                 float eps, int32_t io_dtype, void* stream);

/* Separable D-head read-out with the RMS fused (sca2/arch_sepq.py:93-104 then
 * sca2/ref.py:29-30, the read-out of DHeadSepQ / DHeadSepQPolar.prefill, arch_sepq.py:150):
 * per row r and channel j < dv, n = rsqrt(br^2 + bi^2 + eps_q),
 *   u = [ n (br A + bi Bv) | n (br Bv - bi A) ],   out = u * rsqrt(mean(u^2) + eps)
 * ab (rows, 2, dv) fp32 = [A | Bv] contiguous; br, bi rows of dv fp32 with row stride ld_q
 * (unit column stride); out (rows, 2 dv) fp32 contiguous. */
SCA2_API int sca2_sepq_read_fwd(const float* ab, const float* br, const float* bi, int64_t ld_q,
                       float* out, int64_t rows, int32_t dv, float eps_q, float eps,
                       void* stream);
/* Its gradients from dout (rows, 2 dv): dab (rows, 2, dv) contiguous, dbr / dbi rows of dv
 * with row stride ld_dq. */
SCA2_API int sca2_sepq_read_bwd(const float* ab, const float* br, const float* bi, int64_t ld_q,
                       const float* dout, float* dab, float* dbr, float* dbi, int64_t ld_dq,
                       int64_t rows, int32_t dv, float eps_q, float eps, void* stream);
/* LayerNorm over rows of width d (torch.nn.LayerNorm: biased variance, eps inside the root,
 * affine weight w and bias b), the layers' pre-norms n / fn (sca2/ref.py:345, 352;
 * lapa/layer.py:563, 567) and the LM's final norm (lapa/model.py:37).  fp32 rows, 16-byte
 * aligned; d = 128 ... 1024 in steps of 128 (sca2_layer_norm_supported).  The forward keeps
 * each row's mean and rstd for the backward. */
SCA2_API int sca2_layer_norm_supported(int32_t d);
SCA2_API int sca2_layer_norm_fwd(const float* x, const float* w, const float* b, float* y,
                        float* mean, float* rstd, int64_t rows, int32_t d, float eps,
                        void* stream);
/* Workspace of the backward (floats; the per-CTA partial sums of dw and db). */
SCA2_API size_t sca2_layer_norm_work_floats(int64_t rows, int32_t d);
/* dx (rows, d), and dw, db (d) overwritten (either may be NULL). */
SCA2_API int sca2_layer_norm_bwd(const float* x, const float* w, const float* mean, const float* rstd,
                        const float* dy, float* dx, float* dw, float* db, void* work,
                        int64_t rows, int32_t d, void* stream);
/* RMS read-out of a multi-head read (sca2/arch_gatedc.py:155-156 and _gated_out, :168;
 * lapa/layer.py:384 with H = 1): x rows (rows, H, 2, dvh) contiguous in io_dtype, the heads'
 * [re | im] reads; u rows (rows, 2, H, dvh) fp32 = [re of every head | im of every head] *
 * rsqrt(mean(x^2) + eps).  dvh % 4 == 0; rows 16-byte (fp32) / 8-byte (bf16) aligned. */
SCA2_API int sca2_rms_heads_fwd(const void* x, int32_t io_dtype, float* u, int64_t rows, int32_t H,
                       int32_t dvh, float eps, void* stream);
/* dx (rows, H, 2, dvh) in io_dtype from du (rows, 2, H, dvh) fp32. */
SCA2_API int sca2_rms_heads_bwd(const void* x, int32_t io_dtype, const float* du, void* dx, int64_t rows,
                       int32_t H, int32_t dvh, float eps, void* stream);
/* bf16 hi / lo split of an fp32 matrix x (rows, cols), row stride ld_x: hi = bf16(x),
 * lo = bf16(x - hi).  out (rows, nblk * cols) bf16, row stride ld_out: column block b
 * (b < nblk <= 8) receives lo when bit b of lo_mask is set, else hi.  Operand preparation of
 * the 16-bit projections that replace the heads' fp32 / autocast nn.Linear calls
 * (sca2/arch_sepq.py:94-95: qa_r, qa_i, qb_r, qb_i). */
SCA2_API int sca2_split_bf16(const float* x, int64_t rows, int32_t cols, int64_t ld_x, void* out,
                    int64_t ld_out, int32_t nblk, uint32_t lo_mask, void* stream);

/* ---- projected phases (the fused phase prologue) -------------------------------------------
 * The phase-flavour scan with its phases formed inside the kernels from the head's
 * projections instead of read as phi / psi tensors: a->phw and a->phq then hold K(h) and
 * K(z) (B,T,H,Mh) in `dtype`, and
 *     phi_t = K(h)_t theta + (pos + t) omega,    psi_t = K(z)_t theta + (pos + t) omega
 * in fp32 (each product rounded, then the sum: the expression of LongHead._phase,
 * lapa/layer.py:221-223, and CHeadGated._phases, sca2/arch_gatedc.py:91-95).  Covers the
 * tensor-core path (bf16 values, K = 2 Mh = 64; sca2_scan_proj_supported says whether a call
 * is covered); the projections' rows must be 16-byte aligned. */
typedef struct sca2_phase_proj {
  int32_t dtype;        /* of K(h), K(z) and their gradients: SCA2_F32 or SCA2_BF16 */
  const float* theta;   /* (H, Mh) */
  const float* omega;   /* (H, Mh) */
  const float* pos;     /* device fp32 scalar: position of token 0 (the state's "pos"), or NULL = 0 */
} sca2_phase_proj;

/* 1 if sca2_scan_fwd_proj (training != 0: with chunk states, and sca2_scan_bwd_proj) covers
 * these arguments, else 0. */
SCA2_API int sca2_scan_proj_supported(const sca2_scan_args* a, const sca2_phase_proj* pp,
                   int32_t training);

/* Forward with projected phases; otherwise as sca2_scan_fwd. */
SCA2_API int sca2_scan_fwd_proj(const sca2_scan_args* a, const sca2_phase_proj* pp, sca2_out o,
                   float* S_final, float* chunk_states, void* stream);

/* Bytes of the workspace of sca2_scan_bwd_proj. */
SCA2_API int64_t sca2_scan_proj_work_bytes(int32_t B, int32_t T, int32_t H, int32_t Mh);

/* ---- inference forward with a work buffer ---------------------------------------------------
 * Bytes of the work buffer of sca2_scan_fwd_work for these arguments: B*H*ceil(T/64)*8 KB where
 * the tensor-core forward covers the call at K = 64 (bf16 values), else 0. */
SCA2_API int64_t sca2_scan_fwd_work_bytes(const sca2_scan_args* a);

/* Forward without saved chunk states (inference), with phases (pp NULL, as sca2_scan_fwd with
 * chunk_states NULL) or projected phases (pp non-NULL, as sca2_scan_fwd_proj with chunk_states
 * NULL).  Where sca2_scan_fwd_work_bytes(a) > 0 the delta-rule inverse of every 64-token chunk
 * is first computed chunk-parallel into `work` (16-byte aligned, at least that many bytes), and
 * the sequential chunk walk reads it instead of inverting inside its loop; otherwise `work` is
 * not used.  The outputs agree with the calls named within the bf16 parity bar (the inverse is
 * formed by the same fp32 algorithm and rounded to bf16 in both; its inputs may round in the
 * last bit differently).  Replaces the same reference prefill paths as sca2_scan_fwd
 * (lapa/layer.py:298-366 with no autograd graph kept). */
SCA2_API int sca2_scan_fwd_work(const sca2_scan_args* a, const sca2_phase_proj* pp, sca2_out o,
                   float* S_final, void* work, int64_t work_bytes, void* stream);

/* Backward with projected phases: as sca2_scan_bwd, except that gr->dphw / gr->dphq receive
 * the gradients of K(h) / K(z) in pp->dtype (WRITTEN, not accumulated) and dtheta (H, Mh)
 * the gradient of theta (written). */
SCA2_API int sca2_scan_bwd_proj(const sca2_scan_args* a, const sca2_phase_proj* pp, sca2_out dO,
                   const float* dS_final, const float* chunk_states, const sca2_scan_grads* gr,
                   float* dtheta, void* work, void* stream);

/* ---- D-head diagonal scan ---------------------------------------------------------------
 * Complex diagonal recurrence of the SCA2 D head and its read contracted over M rows:
 *   s_t[m,j] = a_t[m,g(j)] s_{t-1}[m,j] + v_t[j]      g(j) = j / (V/G)
 *   A_t[j]  = mean_m (sr cr + si ci),   Bv_t[j] = mean_m (si cr - sr ci)
 * c = the normalised query per (t,m,j) (DHeadRef, sca2/ref.py:239-275) or, with sep = 1,
 * its separable factor per (t,m) (DHeadSepQ, sca2/arch_sepq.py:100-104).  All tensors fp32
 * and contiguous.  M in {1,2,4,8,16,32}; V/G (channels per gate group) a multiple of 32/M. */
typedef struct sca2_dscan_args {
  int32_t B, T, M, G, V;
  int32_t sep;
  const float* a_re;    /* (B,T,M,G) complex gate */
  const float* a_im;
  const float* v;       /* (B,T,V) */
  const float* c_re;    /* (B,T,M,V), or (B,T,M) with sep */
  const float* c_im;
  const float* S0_re;   /* (B,M,V) incoming state, or NULL = zeros */
  const float* S0_im;
} sca2_dscan_args;

/* Gradients of sca2_dscan_bwd.  da_re, da_im and, with sep, dc_re, dc_im are ACCUMULATED
 * INTO (the caller zero-fills them); dv, dc (without sep) and dS0 are written. */
typedef struct sca2_dscan_grads {
  float* da_re;
  float* da_im;
  float* dv;
  float* dc_re;
  float* dc_im;
  float* dS0_re;        /* or NULL */
  float* dS0_im;
} sca2_dscan_grads;

/* Checkpoint blocks for T tokens: the buffer is (B, sca2_dscan_num_ckpt(T), 2, M, V) fp32. */
SCA2_API int32_t sca2_dscan_num_ckpt(int32_t T);

/* Bytes of the optional device workspace of sca2_dscan_fwd / sca2_dscan_bwd.  With it, a
 * long sequence runs as 16-token blocks in parallel joined by a pass over the blocks; with
 * work = NULL every (b, m, j) runs its T tokens sequentially (same results up to fp32
 * rounding order, far less parallel). */
SCA2_API int64_t sca2_dscan_work_bytes(int32_t B, int32_t T, int32_t M, int32_t G, int32_t V);

/* Forward: ab (B,T,2,V) = [A | Bv] per token; S_re, S_im (B,M,V) the state after T tokens;
 * ckpt NULL, or the checkpoint buffer kept for the backward; work NULL or
 * sca2_dscan_work_bytes of device memory.  T = 1 is the decode step of DHeadRef.step /
 * DHeadSepQ.step (sca2/ref.py:259-275, sca2/arch_sepq.py:152-178). */
SCA2_API int sca2_dscan_fwd(const sca2_dscan_args* a, float* ab, float* S_re, float* S_im,
                   float* ckpt, void* work, void* stream);

/* Backward: dab (B,T,2,V), dS_re / dS_im (B,M,V) or NULL, ckpt as written by the forward,
 * work as for the forward. */
SCA2_API int sca2_dscan_bwd(const sca2_dscan_args* a, const float* dab, const float* dS_re,
                   const float* dS_im, const float* ckpt, const sca2_dscan_grads* g,
                   void* work, void* stream);

/* ---- short head: exact L-tap window read ---------------------------------------------------
 *   phi_t = kh_t theta + ((pos + t) mod L) omega,   psi_t = kz_t theta + ((pos + t) mod L) omega
 *   kappa(t,s) = (1/L) sum_m (wr + i wi)_m exp(i (phi_s - psi_t))
 *   o_t = [ sum_{s=t-L+1..t} Re kappa(t,s) e_s | sum Im kappa(t,s) e_s ]       (B,T,2dv)
 * The write / read / decode of lapa.layer.ShortHead (lapa/layer.py:418-545: _phase :444,
 * _read :450, _banded :488, step :524) and sca2.arch_short.CHeadShort (sca2/arch_short.py:
 * 45-158).  The L-1 previous writes are the ring buffer c0 = cos phi, s0 = sin phi,
 * e0 = value (oldest first).  All tensors fp32, contiguous; 1 <= L <= 32, any dv. */
typedef struct sca2_short_args {
  int32_t B, T, L, dv;
  const int64_t* pos;   /* device scalar: position of token 0 (the state's "pos"), or NULL = 0 */
  const float* kh;      /* (B,T,L) K(h): content of the write phase */
  const float* kz;      /* (B,T,L) K(z): content of the read phase */
  const float* v;       /* (B,T,dv) V(z): the values written */
  const float* theta;   /* (L) */
  const float* omega;   /* (L) the DFT grid 2 pi m / L */
  const float* wr;      /* (L) read weights */
  const float* wi;
  const float* c0;      /* (B,L-1,L) ring buffer, or NULL = init_state (c = 1, s = 0, e = 0) */
  const float* s0;
  const float* e0;      /* (B,L-1,dv) */
} sca2_short_args;

/* Gradients of sca2_short_bwd, all WRITTEN (no zero-fill needed); dc0/ds0/de0 may be NULL. */
typedef struct sca2_short_grads {
  float* dkh;           /* (B,T,L) */
  float* dkz;           /* (B,T,L) */
  float* dv;            /* (B,T,dv) */
  float* dtheta;        /* (L) */
  float* dwr;           /* (L) */
  float* dwi;           /* (L) */
  float* dc0;           /* (B,L-1,L) */
  float* ds0;
  float* de0;           /* (B,L-1,dv) */
} sca2_short_grads;

/* Forward: o (B,T,2dv), or NULL when T = 0; c1, s1 (B,L-1,L) and e1 (B,L-1,dv) the new ring
 * buffer (the last L-1 writes of buffer + call), or NULL to skip it.  Outputs must not alias
 * inputs.  T = 1 is the decode step (ShortHead.step, CHeadShort.step). */
SCA2_API int sca2_short_fwd(const sca2_short_args* a, float* o, float* c1, float* s1, float* e1,
                   void* stream);

/* Bytes of the workspace sca2_short_bwd needs (per-CTA partial sums of the L-vectors). */
SCA2_API int64_t sca2_short_work_bytes(int32_t B, int32_t T, int32_t L, int32_t dv);

/* Backward: dO (B,T,2dv); dc1, ds1, de1 gradients of the new ring buffer or NULL. */
SCA2_API int sca2_short_bwd(const sca2_short_args* a, const float* dO, const float* dc1,
                   const float* ds1, const float* de1, const sca2_short_grads* g, void* work,
                   void* stream);

/* Size of the device array behind sca2_scan_fwd_bwd_noalloc (every GPU that loads the
 * library holds it until the process exits). */
#define SCA2_NOALLOC_SCRATCH_BYTES (16u << 20)

/* Forward + backward in one call that allocates nothing and takes no workspace: for
 * callers that cannot allocate device memory (a plugin inside a runtime that owns the
 * device memory pool, or a path where cudaMalloc must not be called).  No counterpart
 * in the reference.  Same arguments and gradient contract as sca2_scan_fwd followed by
 * sca2_scan_bwd (the per-token and per-head gradient buffers are accumulated into and
 * must be zero-filled by the caller), minus chunk_states: the buffer that the two-call API
 * takes from the caller -- sca2_num_chunks(T) slots of K*V fp32 per (b, h), holding the
 * state entering each chunk, the chunk's saved intermediates and, on the explicit-key
 * K = V = 128 path, the backward's workspace -- lives in a static device array of
 * SCA2_NOALLOC_SCRATCH_BYTES, so B*H*sca2_num_chunks(T)*K*V*4 bytes must fit in it; larger
 * problems return SCA2_ERR_ARG before any launch.  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) and must come before any stream capture.  All calls share the
 * array: calls that overlap on the GPU race and must be serialised. */
SCA2_API int sca2_scan_fwd_bwd_noalloc(const sca2_scan_args* a, sca2_out o, float* S_final,
                                       sca2_out dO, const float* dS_final,
                                       const sca2_scan_grads* gr, void* stream);

/* Read and clear the device fault word of the tensor-core kernels (synchronises the
 * device).  Bit 0: an internal wait on the tensor core timed out; the kernel left early
 * and its outputs are not valid.  Kernels never trap: this word is how a device-side
 * failure reaches the host. */
SCA2_API int sca2_fault_status(uint32_t* faults);

/* Thread-local message of the last failing call on this thread. */
SCA2_API const char* sca2_last_error(void);

/* Library version string. */
SCA2_API const char* sca2_version(void);

#ifdef __cplusplus
}
#endif

#endif /* SCA2B200_H */
