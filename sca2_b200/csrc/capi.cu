// extern "C" entry points of libsca2b200.so: argument validation on the host, then
// dispatch to the kernels.  No entry point allocates memory or synchronises the host.
#include <cstdio>
#include <cstring>
#include <string>

#include "common.cuh"

namespace sca2 {
// scan_f32.cu
int f32_smem_bytes(int K, int R, bool bwd);
int f32_num_chunks(int T);
cudaError_t f32_scan_fwd(const sca2_scan_args& p, const sca2_out& o, float* S_final,
                         float* cstates, cudaStream_t st);
cudaError_t f32_scan_bwd(const sca2_scan_args& p, const sca2_out& dO, const float* dS_final,
                         const float* cstates, const sca2_scan_grads& gr, cudaStream_t st);
// step.cu
int step_rows_per_thread(int K, int V, int vec);
int step_max_rows();
size_t step_smem_bytes(int K, int V, int R, int vec);
cudaError_t launch_step(const sca2_scan_args& p, const float* S_in, float* S_out,
                        const sca2_out& o, int vec, cudaStream_t st);
cudaError_t launch_rms_fwd(const void* x, void* u, int64_t N, int D, float eps, int dt,
                           cudaStream_t st);
cudaError_t launch_rms_bwd(const void* x, const void* du, void* dx, int64_t N, int D, float eps,
                           int dt, cudaStream_t st);
// scan_tc.cu
int tc_fwd_vb(int K, int V, int R, int max_smem);
cudaError_t tc_scan_fwd(const sca2_scan_args& p, int VB, const sca2_out& o, float* S_final,
                        float* cstates, int NCS, cudaStream_t st, const PhaseProj& pp = PhaseProj{},
                        void* work = nullptr);
int64_t tc_infer_work_bytes(const sca2_scan_args& p);
cudaError_t tc_read_faults(unsigned int* out);
cudaError_t tc_read_faults_bwd(unsigned int* out);
// readout.cu
cudaError_t launch_sepq_read_fwd(const float* ab, const float* br, const float* bi, int64_t ldq, float* out,
                                 int64_t rows, int dv, float eps_q, float eps, cudaStream_t st);
cudaError_t launch_sepq_read_bwd(const float* ab, const float* br, const float* bi, int64_t ldq, const float* dout,
                                 float* dab, float* dbr, float* dbi, int64_t lddq, int64_t rows, int dv, float eps_q,
                                 float eps, cudaStream_t st);
cudaError_t launch_split_bf16(const float* x, int64_t rows, int cols, int64_t ldx, void* out, int64_t ldo, int nblk,
                              uint32_t lo_mask, cudaStream_t st);
cudaError_t launch_rms_heads_fwd(const void* x, int dt, float* out, int64_t rows, int H, int dvh, float eps,
                                 cudaStream_t st);
cudaError_t launch_rms_heads_bwd(const void* x, int dt, const float* dout, void* dx, int64_t rows, int H, int dvh,
                                 float eps, cudaStream_t st);
// layernorm.cu
bool ln_supported(int d);
int ln_bwd_parts(int64_t rows);
cudaError_t ln_fwd(const float* x, const float* w, const float* b, float* y, float* mean, float* rstd, int64_t rows,
                   int d, float eps, cudaStream_t st);
cudaError_t ln_bwd(const float* x, const float* w, const float* mean, const float* rstd, const float* dy, float* dx,
                   float* dw, float* db, float* part, int64_t rows, int d, cudaStream_t st);
// dscan.cu
size_t dscan_work_floats(int B, int T, int M, int G, int V);
cudaError_t dscan_fwd(const sca2_dscan_args& p, float* ab, float* S_re, float* S_im, float* ckpt, float* work,
                      cudaStream_t st);
cudaError_t dscan_bwd(const sca2_dscan_args& p, const float* dab, const float* dS_re, const float* dS_im,
                      const float* ckpt, float* work, const sca2_dscan_grads& g, cudaStream_t st);
cudaError_t tc_read_faults_prep(unsigned int* out);
// short.cu
int short_tokens_per_cta(int L, bool bwd, int max_smem);
size_t short_work_floats(int B, int T, int L, int max_smem);
cudaError_t short_fwd(const sca2_short_args& p, float* o, float* c1, float* s1, float* e1, int max_smem,
                      cudaStream_t st);
cudaError_t short_bwd(const sca2_short_args& p, const float* dO, const float* dc1, const float* ds1,
                      const float* de1, const sca2_short_grads& g, float* work, int max_smem, cudaStream_t st);
// scan_tc_bwd.cu
bool tc_train_ok(const sca2_scan_args& p, int max_smem);
cudaError_t tc_scan_bwd(const sca2_scan_args& p, const sca2_out& dO, const float* dS_final, const float* cstates,
                        const sca2_scan_grads& gr, int NCS, cudaStream_t st, const PhaseProj& pp = PhaseProj{});
// gdn_cp.cu
bool cp_covers(const sca2_scan_args& p);
cudaError_t cp_scan_fwd(const sca2_scan_args& p, sca2_out o, float* S_final, float* cstates, int NS,
                        cudaStream_t st);
cudaError_t cp_scan_bwd(const sca2_scan_args& p, sca2_out dO, const float* dS_final, float* cstates,
                        const sca2_scan_grads& gr, int NS, cudaStream_t st);
cudaError_t cp_read_faults(unsigned int* out);
// phase_cp.cu
cudaError_t pcp_read_faults(unsigned int* out);
bool pcp_value_tma(const sca2_scan_args& p, const float* cstates);
// phase_proj.cu
size_t proj_work_floats(int B, int T, int H, int Mh);
cudaError_t proj_bwd(int B, int T, int H, int Mh, int dtype, const float* work, const sca2_tok& kh,
                     const sca2_tok& kz, const float* theta, const sca2_tok& dkh, const sca2_tok& dkz, float* dtheta,
                     cudaStream_t st);
}  // namespace sca2

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(SCA2_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}

int max_optin_smem() {
  int dev = 0, v = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    return 0;
  return v;
}

// Checks shared by the forward, backward and step entry points.
int check_common(const sca2_scan_args* a, bool step) {
  if (!a) return fail(SCA2_ERR_ARG, "null argument struct");
  if (a->flavor != SCA2_FLAVOR_PHASE && a->flavor != SCA2_FLAVOR_KEY)
    return fail(SCA2_ERR_ARG, "flavor must be SCA2_FLAVOR_PHASE or SCA2_FLAVOR_KEY");
  if (a->io_dtype != SCA2_F32 && a->io_dtype != SCA2_BF16)
    return fail(SCA2_ERR_ARG, "io_dtype must be SCA2_F32 or SCA2_BF16");
  if (a->B < 1 || a->H < 1 || a->K < 1 || a->V < 1 || a->T < 0 || (step && a->T != 1))
    return fail(SCA2_ERR_ARG, "sizes must satisfy B, H, K, V >= 1, T >= 0 (T == 1 for a step)");
  if ((int64_t)a->B * a->H > 2147483647LL)
    return fail(SCA2_ERR_ARG, "B * H too large");
  if (a->flavor == SCA2_FLAVOR_PHASE) {
    if (a->K % 2) return fail(SCA2_ERR_ARG, "phase flavour needs an even K (= 2 * Mh)");
    if (!a->wr || !a->wi) return fail(SCA2_ERR_ARG, "phase flavour needs wr and wi");
    if (a->v_times_beta) return fail(SCA2_ERR_ARG, "v_times_beta is a key-flavour option");
  }
  if (a->T > 0 && (!a->phw.ptr || !a->phq.ptr || !a->v.ptr))  // empty inputs may be null
    return fail(SCA2_ERR_ARG, "phw/k, phq/q and v must be non-null");
  if (a->v_times_beta && !a->beta.ptr) return fail(SCA2_ERR_ARG, "v_times_beta needs beta");
  return SCA2_OK;
}

int check_scan(const sca2_scan_args* a, bool bwd) {
  int rc = check_common(a, false);
  if (rc) return rc;
  if (a->K > 128)
    return fail(SCA2_ERR_UNSUPPORTED, "key width K > 128 is not supported by this build");
  const int R = a->flavor == SCA2_FLAVOR_PHASE ? 2 : 1;
  const int need = sca2::f32_smem_bytes(a->K, R, bwd);
  const int have = max_optin_smem();
  if (need > have)
    return fail(SCA2_ERR_UNSUPPORTED, "shape needs " + std::to_string(need) +
                                          " bytes of shared memory per CTA, device allows " +
                                          std::to_string(have));
  return SCA2_OK;
}

}  // namespace

namespace sca2 {
// Lets the other entry-point files report through sca2_last_error().
void set_last_error(const std::string& msg) { g_err = msg; }
}  // namespace sca2

extern "C" {

const char* sca2_last_error(void) { return g_err.c_str(); }

const char* sca2_version(void) { return "sca2b200 0.1.0 (sm_100a)"; }

int sca2_fault_status(uint32_t* faults) {
  if (!faults) return fail(SCA2_ERR_ARG, "null output");
  unsigned int f = 0;
  unsigned int fb = 0, fp = 0, fc = 0, fq = 0;
  cudaError_t e = sca2::tc_read_faults(&f);
  if (e == cudaSuccess) e = sca2::tc_read_faults_bwd(&fb);
  if (e == cudaSuccess) e = sca2::tc_read_faults_prep(&fp);
  if (e == cudaSuccess) e = sca2::cp_read_faults(&fc);
  if (e == cudaSuccess) e = sca2::pcp_read_faults(&fq);
  if (e != cudaSuccess) return cuda_fail(e, "sca2_fault_status");
  *faults = f | fb | fp | fc | fq;
  return SCA2_OK;
}

int32_t sca2_num_chunks(int32_t T) { return T > 0 ? sca2::state_slots(T) : 0; }

int sca2_scan_value_tma(const sca2_scan_args* a) {
  if (!a || check_scan(a, false) != SCA2_OK) return 0;
  // any 16-byte aligned address stands for the caller's chunk-state buffer
  return sca2::pcp_value_tma(*a, reinterpret_cast<const float*>(static_cast<uintptr_t>(256))) ? 1 : 0;
}

int sca2_scan_fwd(const sca2_scan_args* a, sca2_out o, float* S_final, float* chunk_states,
                  void* stream) {
  int rc = check_scan(a, false);
  if (rc) return rc;
  if (!o.ptr && a->T > 0) return fail(SCA2_ERR_ARG, "output o must be non-null");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const size_t sbytes = (size_t)a->B * a->H * a->K * a->V * sizeof(float);
  if (a->T == 0) {  // empty input: the state passes through unchanged
    if (S_final) {
      cudaError_t e = a->S0 ? cudaMemcpyAsync(S_final, a->S0, sbytes, cudaMemcpyDeviceToDevice, st)
                            : cudaMemsetAsync(S_final, 0, sbytes, st);
      if (e != cudaSuccess) return cuda_fail(e, "sca2_scan_fwd(T=0)");
    }
    return SCA2_OK;
  }
  // training of the explicit-key form at K = V = 128: chunk-parallel tensor-core path
  if (chunk_states && sca2::cp_covers(*a)) {
    cudaError_t e = sca2::cp_scan_fwd(*a, o, S_final, chunk_states, sca2::state_slots(a->T), st);
    if (e != cudaSuccess) return cuda_fail(e, "sca2_scan_fwd");
    return SCA2_OK;
  }
  // bf16 runs on the tensor cores when the shape is covered; with saved chunk states (training)
  // only where the tensor-core backward covers the shape too, so the pair stays consistent
  const int R = a->flavor == SCA2_FLAVOR_PHASE ? 2 : 1;
  const int smem = max_optin_smem();
  int vb = 0;
  if (a->io_dtype == SCA2_BF16) {
    if (!chunk_states) vb = sca2::tc_fwd_vb(a->K, a->V, R, smem);
    else if (sca2::tc_train_ok(*a, smem)) vb = sca2::tc_fwd_vb(a->K, a->V, R, smem);
  }
  cudaError_t e = vb ? sca2::tc_scan_fwd(*a, vb, o, S_final, chunk_states, sca2::state_slots(a->T), st)
                     : sca2::f32_scan_fwd(*a, o, S_final, chunk_states, st);
  if (e != cudaSuccess) return cuda_fail(e, "sca2_scan_fwd");
  return SCA2_OK;
}

static bool tok_dense(const sca2_tok& t, const sca2_scan_args* a, int C) {
  return t.sh == C && t.st == (int64_t)a->H * C && t.sb == (int64_t)a->T * a->H * C;
}

// Overwrite mode: zero the gradients the kernels accumulate into.  The per-token key-side rows
// are left alone when the tensor-core backward writes them itself (one CTA per (b, h)).
static cudaError_t init_grads(const sca2_scan_args* a, const sca2_scan_grads* gr, bool rows_written,
                              cudaStream_t st) {
  const int KH = a->flavor == SCA2_FLAVOR_PHASE ? a->K / 2 : a->K;
  const size_t tok = (size_t)a->B * a->T * a->H * sizeof(float);
  cudaError_t e = cudaSuccess;
  auto z = [&](const void* p, size_t bytes) {
    if (p && bytes && e == cudaSuccess) e = cudaMemsetAsync(const_cast<void*>(p), 0, bytes, st);
  };
  if (!rows_written) {
    z(gr->dphw.ptr, tok * KH);
    z(gr->dphq.ptr, tok * KH);
  }
  if (a->beta.ptr) z(gr->dbeta.ptr, tok);
  if (a->g.ptr) z(gr->dg.ptr, tok);
  if (a->lam) z(gr->dlam, (size_t)a->H * KH * sizeof(float));
  if (a->flavor == SCA2_FLAVOR_PHASE) {
    z(gr->dwr, (size_t)a->H * KH * sizeof(float));
    z(gr->dwi, (size_t)a->H * KH * sizeof(float));
  }
  return e;
}

static int check_overwrite(const sca2_scan_args* a, const sca2_scan_grads* gr) {
  const int KH = a->flavor == SCA2_FLAVOR_PHASE ? a->K / 2 : a->K;
  if (!tok_dense(gr->dphw, a, KH) || !tok_dense(gr->dphq, a, KH) ||
      (a->beta.ptr && !tok_dense(gr->dbeta, a, 1)) || (a->g.ptr && !tok_dense(gr->dg, a, 1)))
    return fail(SCA2_ERR_ARG, "overwrite mode needs dense (B,T,H,C) gradient tensors");
  return SCA2_OK;
}

// whether the tensor-core backward writes the key-side rows itself in overwrite mode
static bool tc_rows_written(const sca2_scan_args* a, const sca2_tok& dphw, const sca2_tok& dphq) {
  auto a16 = [](const void* q) { return ((uintptr_t)q & 15u) == 0; };
  return a->V == 64 && a16(dphw.ptr) && a16(dphq.ptr) && dphw.sb % 4 == 0 && dphw.st % 4 == 0 &&
         dphw.sh % 4 == 0 && dphq.sb % 4 == 0 && dphq.st % 4 == 0 && dphq.sh % 4 == 0;
}

int sca2_scan_bwd(const sca2_scan_args* a, sca2_out dO, const float* dS_final,
                  float* chunk_states, const sca2_scan_grads* gr, void* stream) {
  int rc = check_scan(a, true);
  if (rc) return rc;
  if (!gr) return fail(SCA2_ERR_ARG, "null gradient struct");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const size_t sbytes = (size_t)a->B * a->H * a->K * a->V * sizeof(float);
  if (a->T == 0) {
    if (gr->dS0) {
      cudaError_t e = dS_final
                          ? cudaMemcpyAsync(gr->dS0, dS_final, sbytes, cudaMemcpyDeviceToDevice, st)
                          : cudaMemsetAsync(gr->dS0, 0, sbytes, st);
      if (e != cudaSuccess) return cuda_fail(e, "sca2_scan_bwd(T=0)");
    }
    return SCA2_OK;
  }
  if (!dO.ptr || !chunk_states) return fail(SCA2_ERR_ARG, "dO and chunk_states must be non-null");
  if (!gr->dphw.ptr || !gr->dphq.ptr || !gr->dv.ptr)
    return fail(SCA2_ERR_ARG, "dphw/dk, dphq/dq and dv must be non-null");
  if (a->beta.ptr && !gr->dbeta.ptr) return fail(SCA2_ERR_ARG, "beta given but dbeta is null");
  if (a->g.ptr && !gr->dg.ptr) return fail(SCA2_ERR_ARG, "g given but dg is null");
  if (sca2::cp_covers(*a)) {  // the chunk-parallel path (its forward saved the chunk data)
    auto a16 = [](const void* q) { return ((uintptr_t)q & 15u) == 0; };
    const int64_t q = gr->grad_io_dtype ? 8 : 4;  // elements per 16 bytes
    auto rows = [&](const sca2_tok& t) { return a16(t.ptr) && t.sb % q == 0 && t.st % q == 0 && t.sh % q == 0; };
    if (!rows(gr->dphw) || !rows(gr->dphq))
      return fail(SCA2_ERR_ARG, "dk and dq rows must be 16-byte aligned for K = V = 128 explicit-key training");
    if (gr->grad_io_dtype && !gr->overwrite)
      return fail(SCA2_ERR_UNSUPPORTED, "dk / dq in the io dtype are written, not accumulated (set overwrite)");
    if (gr->overwrite && (rc = check_overwrite(a, gr))) return rc;
    cudaError_t e = sca2::cp_scan_bwd(*a, dO, dS_final, chunk_states, *gr,
                                      sca2::state_slots(a->T), st);
    if (e != cudaSuccess) return cuda_fail(e, "sca2_scan_bwd");
    return SCA2_OK;
  }
  if (gr->grad_io_dtype)
    return fail(SCA2_ERR_UNSUPPORTED, "dk / dq in the io dtype need explicit-key bf16 training at K = V = 128 "
                                      "without lam (16-byte aligned rows)");
  const bool tc = sca2::tc_train_ok(*a, max_optin_smem());
  if (gr->overwrite) {
    if ((rc = check_overwrite(a, gr))) return rc;
    cudaError_t e = init_grads(a, gr, tc && tc_rows_written(a, gr->dphw, gr->dphq), st);
    if (e != cudaSuccess) return cuda_fail(e, "sca2_scan_bwd(init)");
  }
  cudaError_t e = tc ? sca2::tc_scan_bwd(*a, dO, dS_final, chunk_states, *gr, sca2::state_slots(a->T), st)
                     : sca2::f32_scan_bwd(*a, dO, dS_final, chunk_states, *gr, st);
  if (e != cudaSuccess) return cuda_fail(e, "sca2_scan_bwd");
  return SCA2_OK;
}

static bool proj_rows_ok(const sca2_tok& t, int dtype) {
  const int64_t q = dtype == SCA2_BF16 ? 8 : 4;  // elements per 16 bytes
  return t.ptr && ((uintptr_t)t.ptr & 15u) == 0 && t.sb % q == 0 && t.st % q == 0 && t.sh % q == 0;
}

static bool proj_covered(const sca2_scan_args* a, const sca2_phase_proj* pp, bool training) {
  if (!a || !pp || a->flavor != SCA2_FLAVOR_PHASE || a->io_dtype != SCA2_BF16 || a->K != 64) return false;
  if (pp->dtype != SCA2_F32 && pp->dtype != SCA2_BF16) return false;
  if (!pp->theta || !pp->omega || !proj_rows_ok(a->phw, pp->dtype) || !proj_rows_ok(a->phq, pp->dtype)) return false;
  const int smem = max_optin_smem();
  if (training) return sca2::tc_train_ok(*a, smem) && sca2::tc_fwd_vb(a->K, a->V, 2, smem) > 0;
  return sca2::tc_fwd_vb(a->K, a->V, 2, smem) > 0;
}

static sca2::PhaseProj to_pp(const sca2_phase_proj* pp) {
  return sca2::PhaseProj{1, pp->dtype, pp->theta, pp->omega, pp->pos};
}

int sca2_scan_proj_supported(const sca2_scan_args* a, const sca2_phase_proj* pp, int32_t training) {
  return (check_scan(a, training != 0) == SCA2_OK && proj_covered(a, pp, training != 0)) ? 1 : 0;
}

int sca2_scan_fwd_proj(const sca2_scan_args* a, const sca2_phase_proj* pp, sca2_out o, float* S_final,
                       float* chunk_states, void* stream) {
  int rc = check_scan(a, false);
  if (rc) return rc;
  if (a->T == 0) return sca2_scan_fwd(a, o, S_final, chunk_states, stream);
  if (!o.ptr) return fail(SCA2_ERR_ARG, "output o must be non-null");
  if (!proj_covered(a, pp, chunk_states != nullptr))
    return fail(SCA2_ERR_UNSUPPORTED, "projected phases need the tensor-core path (bf16 values, K = 64) and "
                                      "16-byte aligned projection rows");
  const int vb = sca2::tc_fwd_vb(a->K, a->V, 2, max_optin_smem());
  cudaError_t e = sca2::tc_scan_fwd(*a, vb, o, S_final, chunk_states, sca2::state_slots(a->T),
                                    reinterpret_cast<cudaStream_t>(stream), to_pp(pp));
  if (e != cudaSuccess) return cuda_fail(e, "sca2_scan_fwd_proj");
  return SCA2_OK;
}

// Inference forward with a caller work buffer: where the tensor-core forward covers the call at
// K = 64, T of every chunk is computed chunk-parallel into the work buffer first, so the chunk walk
// no longer inverts inside its sequential loop.  Needs sca2_scan_fwd_work_bytes(a) bytes; 0 bytes
// (any other shape or dtype) runs exactly what sca2_scan_fwd / sca2_scan_fwd_proj run without
// saved chunk states.
int64_t sca2_scan_fwd_work_bytes(const sca2_scan_args* a) {
  if (!a || check_scan(a, false) != SCA2_OK || a->T <= 0 || a->io_dtype != SCA2_BF16) return 0;
  const int R = a->flavor == SCA2_FLAVOR_PHASE ? 2 : 1;
  if (sca2::tc_fwd_vb(a->K, a->V, R, max_optin_smem()) == 0) return 0;
  return sca2::tc_infer_work_bytes(*a);
}

int sca2_scan_fwd_work(const sca2_scan_args* a, const sca2_phase_proj* pp, sca2_out o, float* S_final, void* work,
                       int64_t work_bytes, void* stream) {
  int rc = check_scan(a, false);
  if (rc) return rc;
  if (a->T == 0) return sca2_scan_fwd(a, o, S_final, nullptr, stream);
  if (!o.ptr) return fail(SCA2_ERR_ARG, "output o must be non-null");
  if (pp && !proj_covered(a, pp, false))
    return fail(SCA2_ERR_UNSUPPORTED, "projected phases need the tensor-core path (bf16 values, K = 64) and "
                                      "16-byte aligned projection rows");
  const int64_t need = sca2_scan_fwd_work_bytes(a);
  if (need > 0 && (!work || work_bytes < need))
    return fail(SCA2_ERR_ARG, "work buffer smaller than sca2_scan_fwd_work_bytes()");
  if (need > 0 && ((uintptr_t)work & 15u) != 0) return fail(SCA2_ERR_ARG, "work buffer not 16-byte aligned");
  if (need == 0) return pp ? sca2_scan_fwd_proj(a, pp, o, S_final, nullptr, stream)
                           : sca2_scan_fwd(a, o, S_final, nullptr, stream);
  const int R = a->flavor == SCA2_FLAVOR_PHASE ? 2 : 1;
  const int vb = sca2::tc_fwd_vb(a->K, a->V, R, max_optin_smem());
  cudaError_t e = sca2::tc_scan_fwd(*a, vb, o, S_final, nullptr, sca2::state_slots(a->T),
                                    reinterpret_cast<cudaStream_t>(stream),
                                    pp ? to_pp(pp) : sca2::PhaseProj{}, work);
  if (e != cudaSuccess) return cuda_fail(e, "sca2_scan_fwd_work");
  return SCA2_OK;
}

int64_t sca2_scan_proj_work_bytes(int32_t B, int32_t T, int32_t H, int32_t Mh) {
  if (B < 1 || T < 1 || H < 1 || Mh < 1) return 0;
  return (int64_t)(sca2::proj_work_floats(B, T, H, Mh) * sizeof(float));
}

int sca2_scan_bwd_proj(const sca2_scan_args* a, const sca2_phase_proj* pp, sca2_out dO, const float* dS_final,
                       const float* chunk_states, const sca2_scan_grads* gr, float* dtheta, void* work,
                       void* stream) {
  int rc = check_scan(a, true);
  if (rc) return rc;
  if (!gr || !dtheta) return fail(SCA2_ERR_ARG, "null gradient struct or dtheta");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int Mh = a->K / 2;
  if (a->T == 0) {
    cudaError_t e = cudaMemsetAsync(dtheta, 0, (size_t)a->H * Mh * sizeof(float), st);
    if (e != cudaSuccess) return cuda_fail(e, "sca2_scan_bwd_proj(T=0)");
    // T = 0 reads and writes no chunk state
    return sca2_scan_bwd(a, dO, dS_final, const_cast<float*>(chunk_states), gr, stream);
  }
  if (!dO.ptr || !chunk_states || !work) return fail(SCA2_ERR_ARG, "dO, chunk_states and work must be non-null");
  if (!proj_covered(a, pp, true) || !proj_rows_ok(gr->dphw, pp->dtype) || !proj_rows_ok(gr->dphq, pp->dtype))
    return fail(SCA2_ERR_UNSUPPORTED, "projected phases need the tensor-core path (bf16 values, K = 64) and "
                                      "16-byte aligned projection rows");
  if (!gr->dv.ptr) return fail(SCA2_ERR_ARG, "dv must be non-null");
  if (a->beta.ptr && !gr->dbeta.ptr) return fail(SCA2_ERR_ARG, "beta given but dbeta is null");
  if (a->g.ptr && !gr->dg.ptr) return fail(SCA2_ERR_ARG, "g given but dg is null");
  // d(phi), d(psi) into the workspace (written by the kernel when one CTA owns each row, else
  // zero-filled and accumulated into), then the projections' gradients
  float* w = static_cast<float*>(work);
  const size_t n = (size_t)a->B * a->T * a->H * Mh;
  sca2_scan_grads g2 = *gr;
  const int64_t sh = Mh, stt = (int64_t)a->H * Mh, sb = (int64_t)a->T * stt;
  g2.dphw = sca2_tok{w, sb, stt, sh};
  g2.dphq = sca2_tok{w + n, sb, stt, sh};
  g2.overwrite = tc_rows_written(a, g2.dphw, g2.dphq) ? 1 : 0;
  cudaError_t e = g2.overwrite ? cudaSuccess : cudaMemsetAsync(w, 0, 2 * n * sizeof(float), st);
  if (e == cudaSuccess && gr->overwrite) {
    if ((rc = check_overwrite(a, &g2))) return rc;
    e = init_grads(a, &g2, true, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "sca2_scan_bwd_proj");
  e = sca2::tc_scan_bwd(*a, dO, dS_final, chunk_states, g2, sca2::state_slots(a->T), st, to_pp(pp));
  if (e == cudaSuccess)
    e = sca2::proj_bwd(a->B, a->T, a->H, Mh, pp->dtype, w, a->phw, a->phq, pp->theta, gr->dphw, gr->dphq, dtheta, st);
  if (e != cudaSuccess) return cuda_fail(e, "sca2_scan_bwd_proj");
  return SCA2_OK;
}

int sca2_scan_step(const sca2_scan_args* a, const float* S_in, float* S_out, sca2_out o,
                   void* stream) {
  int rc = check_common(a, true);
  if (rc) return rc;
  if (!S_in || !S_out || !o.ptr) return fail(SCA2_ERR_ARG, "S_in, S_out and o must be non-null");
  const int vec = (a->V % 4 == 0 && ((uintptr_t)S_in % 16 == 0) && ((uintptr_t)S_out % 16 == 0)) ? 4 : 1;
  const int rows = sca2::step_rows_per_thread(a->K, a->V, vec);
  if (rows > sca2::step_max_rows())
    return fail(SCA2_ERR_UNSUPPORTED, "state too large for the decode kernel (K*V)");
  const int R = a->flavor == SCA2_FLAVOR_PHASE ? 2 : 1;
  if ((int)sca2::step_smem_bytes(a->K, a->V, R, vec) > max_optin_smem())
    return fail(SCA2_ERR_UNSUPPORTED, "decode step needs too much shared memory");
  cudaError_t e = sca2::launch_step(*a, S_in, S_out, o, vec, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "sca2_scan_step");
  return SCA2_OK;
}

static int check_dscan(const sca2_dscan_args* a) {
  if (!a) return fail(SCA2_ERR_ARG, "null dscan args");
  if (a->B < 1 || a->T < 0 || a->G < 1 || a->V < 1) return fail(SCA2_ERR_ARG, "dscan: bad sizes");
  if (a->M != 1 && a->M != 2 && a->M != 4 && a->M != 8 && a->M != 16 && a->M != 32)
    return fail(SCA2_ERR_UNSUPPORTED, "dscan: M must be a power of two <= 32");
  if (a->V % a->G) return fail(SCA2_ERR_ARG, "dscan: V must be a multiple of G");
  const int gs = a->V / a->G, jw = 32 / a->M;
  if (gs % jw) return fail(SCA2_ERR_UNSUPPORTED, "dscan: channels per gate group must be a multiple of 32/M");
  if (a->T > 0 && (!a->a_re || !a->a_im || !a->v || !a->c_re || !a->c_im))
    return fail(SCA2_ERR_ARG, "dscan: null input");
  if ((a->S0_re == nullptr) != (a->S0_im == nullptr)) return fail(SCA2_ERR_ARG, "dscan: S0 needs both parts");
  return SCA2_OK;
}

int32_t sca2_dscan_num_ckpt(int32_t T) { return T > 0 ? (T + 15) / 16 : 0; }

int64_t sca2_dscan_work_bytes(int32_t B, int32_t T, int32_t M, int32_t G, int32_t V) {
  if (B < 1 || T < 1 || M < 1 || G < 1 || V < 1) return 0;
  return (int64_t)(sca2::dscan_work_floats(B, T, M, G, V) * sizeof(float));
}

int sca2_dscan_fwd(const sca2_dscan_args* a, float* ab, float* S_re, float* S_im, float* ckpt, void* work,
                   void* stream) {
  int rc = check_dscan(a);
  if (rc) return rc;
  if (!S_re || !S_im || (a->T > 0 && !ab)) return fail(SCA2_ERR_ARG, "dscan: null output");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (a->T == 0) {
    const size_t n = (size_t)a->B * a->M * a->V * sizeof(float);
    cudaError_t e = a->S0_re ? cudaMemcpyAsync(S_re, a->S0_re, n, cudaMemcpyDeviceToDevice, st)
                             : cudaMemsetAsync(S_re, 0, n, st);
    if (e == cudaSuccess)
      e = a->S0_im ? cudaMemcpyAsync(S_im, a->S0_im, n, cudaMemcpyDeviceToDevice, st) : cudaMemsetAsync(S_im, 0, n, st);
    if (e != cudaSuccess) return cuda_fail(e, "sca2_dscan_fwd(T=0)");
    return SCA2_OK;
  }
  cudaError_t e = sca2::dscan_fwd(*a, ab, S_re, S_im, ckpt, static_cast<float*>(work), st);
  if (e != cudaSuccess) return cuda_fail(e, "sca2_dscan_fwd");
  return SCA2_OK;
}

int sca2_dscan_bwd(const sca2_dscan_args* a, const float* dab, const float* dS_re, const float* dS_im,
                   const float* ckpt, const sca2_dscan_grads* g, void* work, void* stream) {
  int rc = check_dscan(a);
  if (rc) return rc;
  if (!g) return fail(SCA2_ERR_ARG, "dscan: null gradient struct");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (a->T == 0) {
    const size_t n = (size_t)a->B * a->M * a->V * sizeof(float);
    cudaError_t e = cudaSuccess;
    if (g->dS0_re) e = dS_re ? cudaMemcpyAsync(g->dS0_re, dS_re, n, cudaMemcpyDeviceToDevice, st) : cudaMemsetAsync(g->dS0_re, 0, n, st);
    if (e == cudaSuccess && g->dS0_im)
      e = dS_im ? cudaMemcpyAsync(g->dS0_im, dS_im, n, cudaMemcpyDeviceToDevice, st) : cudaMemsetAsync(g->dS0_im, 0, n, st);
    if (e != cudaSuccess) return cuda_fail(e, "sca2_dscan_bwd(T=0)");
    return SCA2_OK;
  }
  if (!dab || !ckpt || !g->da_re || !g->da_im || !g->dv || !g->dc_re || !g->dc_im)
    return fail(SCA2_ERR_ARG, "dscan: dab, ckpt and gradient buffers must be non-null");
  cudaError_t e = sca2::dscan_bwd(*a, dab, dS_re, dS_im, ckpt, static_cast<float*>(work), *g, st);
  if (e != cudaSuccess) return cuda_fail(e, "sca2_dscan_bwd");
  return SCA2_OK;
}

int sca2_rms_fwd(const void* x, void* u, int64_t N, int32_t D, float eps, int32_t io_dtype,
                 void* stream) {
  if (!x || !u || N < 0 || D < 1) return fail(SCA2_ERR_ARG, "rms: bad arguments");
  if (io_dtype != SCA2_F32 && io_dtype != SCA2_BF16) return fail(SCA2_ERR_ARG, "rms: bad dtype");
  if (N == 0) return SCA2_OK;
  cudaError_t e = sca2::launch_rms_fwd(x, u, N, D, eps, io_dtype, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "sca2_rms_fwd");
  return SCA2_OK;
}

int sca2_rms_bwd(const void* x, const void* du, void* dx, int64_t N, int32_t D, float eps,
                 int32_t io_dtype, void* stream) {
  if (!x || !du || !dx || N < 0 || D < 1) return fail(SCA2_ERR_ARG, "rms: bad arguments");
  if (io_dtype != SCA2_F32 && io_dtype != SCA2_BF16) return fail(SCA2_ERR_ARG, "rms: bad dtype");
  if (N == 0) return SCA2_OK;
  cudaError_t e = sca2::launch_rms_bwd(x, du, dx, N, D, eps, io_dtype, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "sca2_rms_bwd");
  return SCA2_OK;
}

int sca2_sepq_read_fwd(const float* ab, const float* br, const float* bi, int64_t ld_q, float* out, int64_t rows,
                       int32_t dv, float eps_q, float eps, void* stream) {
  if (rows < 0 || dv < 1 || ld_q < dv) return fail(SCA2_ERR_ARG, "sepq_read: bad sizes");
  if (rows == 0) return SCA2_OK;
  if (!ab || !br || !bi || !out) return fail(SCA2_ERR_ARG, "sepq_read: null pointer");
  cudaError_t e = sca2::launch_sepq_read_fwd(ab, br, bi, ld_q, out, rows, dv, eps_q, eps,
                                             reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "sca2_sepq_read_fwd");
  return SCA2_OK;
}

int sca2_sepq_read_bwd(const float* ab, const float* br, const float* bi, int64_t ld_q, const float* dout,
                       float* dab, float* dbr, float* dbi, int64_t ld_dq, int64_t rows, int32_t dv, float eps_q,
                       float eps, void* stream) {
  if (rows < 0 || dv < 1 || ld_q < dv || ld_dq < dv) return fail(SCA2_ERR_ARG, "sepq_read: bad sizes");
  if (rows == 0) return SCA2_OK;
  if (!ab || !br || !bi || !dout || !dab || !dbr || !dbi) return fail(SCA2_ERR_ARG, "sepq_read: null pointer");
  cudaError_t e = sca2::launch_sepq_read_bwd(ab, br, bi, ld_q, dout, dab, dbr, dbi, ld_dq, rows, dv, eps_q, eps,
                                             reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "sca2_sepq_read_bwd");
  return SCA2_OK;
}

int sca2_layer_norm_supported(int32_t d) { return sca2::ln_supported(d) ? 1 : 0; }

size_t sca2_layer_norm_work_floats(int64_t rows, int32_t d) {
  return rows > 0 && sca2::ln_supported(d) ? (size_t)sca2::ln_bwd_parts(rows) * 2 * (size_t)d : 0;
}

static int check_ln(const void* x, const void* w, int64_t rows, int32_t d) {
  if (rows < 0) return fail(SCA2_ERR_ARG, "layer_norm: bad sizes");
  if (!sca2::ln_supported(d)) return fail(SCA2_ERR_UNSUPPORTED, "layer_norm: width must be 128 ... 1024 in steps of 128");
  if (rows > 0 && (!x || !w)) return fail(SCA2_ERR_ARG, "layer_norm: null pointer");
  if (((uintptr_t)x | (uintptr_t)w) & 15u) return fail(SCA2_ERR_ARG, "layer_norm: rows must be 16-byte aligned");
  return SCA2_OK;
}

int sca2_layer_norm_fwd(const float* x, const float* w, const float* b, float* y, float* mean, float* rstd,
                        int64_t rows, int32_t d, float eps, void* stream) {
  if (int r = check_ln(x, w, rows, d)) return r;
  if (rows == 0) return SCA2_OK;
  if (!b || !y || !mean || !rstd || (((uintptr_t)b | (uintptr_t)y) & 15u))
    return fail(SCA2_ERR_ARG, "layer_norm: null or misaligned output");
  cudaError_t e = sca2::ln_fwd(x, w, b, y, mean, rstd, rows, d, eps, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "sca2_layer_norm_fwd");
  return SCA2_OK;
}

int sca2_layer_norm_bwd(const float* x, const float* w, const float* mean, const float* rstd, const float* dy,
                        float* dx, float* dw, float* db, void* work, int64_t rows, int32_t d, void* stream) {
  if (int r = check_ln(x, w, rows, d)) return r;
  if (rows == 0) return SCA2_OK;
  if (!mean || !rstd || !dy || !dx || !work || (((uintptr_t)dy | (uintptr_t)dx) & 15u))
    return fail(SCA2_ERR_ARG, "layer_norm: null or misaligned argument");
  cudaError_t e = sca2::ln_bwd(x, w, mean, rstd, dy, dx, dw, db, reinterpret_cast<float*>(work), rows, d,
                               reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "sca2_layer_norm_bwd");
  return SCA2_OK;
}

static int check_rms_heads(const void* x, const void* y, int64_t rows, int32_t H, int32_t dvh, int32_t io_dtype) {
  if (rows < 0 || H < 1 || dvh < 4 || dvh % 4) return fail(SCA2_ERR_ARG, "rms_heads: bad sizes (dvh % 4 != 0?)");
  if (io_dtype != SCA2_F32 && io_dtype != SCA2_BF16) return fail(SCA2_ERR_ARG, "rms_heads: bad dtype");
  if (rows > 0 && (!x || !y)) return fail(SCA2_ERR_ARG, "rms_heads: null pointer");
  const uintptr_t a = io_dtype == SCA2_BF16 ? 8 : 16;
  if (((uintptr_t)x % a) || ((uintptr_t)y % 16)) return fail(SCA2_ERR_ARG, "rms_heads: misaligned rows");
  return SCA2_OK;
}

int sca2_rms_heads_fwd(const void* x, int32_t io_dtype, float* u, int64_t rows, int32_t H, int32_t dvh, float eps,
                       void* stream) {
  if (int r = check_rms_heads(x, u, rows, H, dvh, io_dtype)) return r;
  if (rows == 0) return SCA2_OK;
  cudaError_t e = sca2::launch_rms_heads_fwd(x, io_dtype, u, rows, H, dvh, eps, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "sca2_rms_heads_fwd");
  return SCA2_OK;
}

int sca2_rms_heads_bwd(const void* x, int32_t io_dtype, const float* du, void* dx, int64_t rows, int32_t H,
                       int32_t dvh, float eps, void* stream) {
  if (int r = check_rms_heads(x, du, rows, H, dvh, io_dtype)) return r;
  if (rows > 0 && (!dx || ((uintptr_t)dx % (io_dtype == SCA2_BF16 ? 8 : 16))))
    return fail(SCA2_ERR_ARG, "rms_heads: null or misaligned dx");
  if (rows == 0) return SCA2_OK;
  cudaError_t e =
      sca2::launch_rms_heads_bwd(x, io_dtype, du, dx, rows, H, dvh, eps, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "sca2_rms_heads_bwd");
  return SCA2_OK;
}

int sca2_split_bf16(const float* x, int64_t rows, int32_t cols, int64_t ld_x, void* out, int64_t ld_out,
                    int32_t nblk, uint32_t lo_mask, void* stream) {
  if (rows < 0 || cols < 1 || ld_x < cols || nblk < 1 || nblk > 8 || ld_out < (int64_t)nblk * cols)
    return fail(SCA2_ERR_ARG, "split_bf16: bad sizes");
  if (rows == 0) return SCA2_OK;
  if (!x || !out) return fail(SCA2_ERR_ARG, "split_bf16: null pointer");
  cudaError_t e = sca2::launch_split_bf16(x, rows, cols, ld_x, out, ld_out, nblk, lo_mask,
                                          reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "sca2_split_bf16");
  return SCA2_OK;
}

static int check_short(const sca2_short_args* a) {
  if (!a) return fail(SCA2_ERR_ARG, "null short-head args");
  if (a->B < 1 || a->T < 0 || a->L < 1 || a->dv < 1) return fail(SCA2_ERR_ARG, "short: bad sizes");
  if (a->L > 32) return fail(SCA2_ERR_UNSUPPORTED, "short: window L must be <= 32");
  if (a->T > (1 << 27) - 64) return fail(SCA2_ERR_UNSUPPORTED, "short: T must be below 2^27 - 64");
  if (a->T > 0 && (!a->kh || !a->kz || !a->v)) return fail(SCA2_ERR_ARG, "short: null input");
  if (!a->theta || !a->omega || !a->wr || !a->wi) return fail(SCA2_ERR_ARG, "short: null parameter");
  if ((a->c0 == nullptr) != (a->s0 == nullptr)) return fail(SCA2_ERR_ARG, "short: c0 and s0 go together");
  if (sca2::short_tokens_per_cta(a->L, true, max_optin_smem()) == 0)
    return fail(SCA2_ERR_UNSUPPORTED, "short: window too large for shared memory");
  return SCA2_OK;
}

int sca2_short_fwd(const sca2_short_args* a, float* o, float* c1, float* s1, float* e1, void* stream) {
  int rc = check_short(a);
  if (rc) return rc;
  if (a->T > 0 && !o) return fail(SCA2_ERR_ARG, "short: null output");
  if ((c1 == nullptr) != (s1 == nullptr) || (c1 == nullptr) != (e1 == nullptr))
    return fail(SCA2_ERR_ARG, "short: pass all of c1, s1, e1 or none");
  cudaError_t e = sca2::short_fwd(*a, o, c1, s1, e1, max_optin_smem(), reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "sca2_short_fwd");
  return SCA2_OK;
}

int64_t sca2_short_work_bytes(int32_t B, int32_t T, int32_t L, int32_t dv) {
  if (B < 1 || T < 1 || L < 1 || L > 32 || dv < 1) return 0;
  return (int64_t)(sca2::short_work_floats(B, T, L, max_optin_smem()) * sizeof(float));
}

int sca2_short_bwd(const sca2_short_args* a, const float* dO, const float* dc1, const float* ds1,
                   const float* de1, const sca2_short_grads* g, void* work, void* stream) {
  int rc = check_short(a);
  if (rc) return rc;
  if (!g || !g->dtheta || !g->dwr || !g->dwi) return fail(SCA2_ERR_ARG, "short: null gradient buffer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int n = a->L - 1;
  if (a->T == 0) {  // the new buffer is the old one
    cudaError_t e = cudaSuccess;
    const size_t nl = (size_t)a->B * n * a->L * sizeof(float), nd = (size_t)a->B * n * a->dv * sizeof(float);
    auto pass = [&](float* dst, const float* src, size_t bytes) {
      if (dst && e == cudaSuccess && bytes)
        e = src ? cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, st) : cudaMemsetAsync(dst, 0, bytes, st);
    };
    pass(g->dc0, dc1, nl);
    pass(g->ds0, ds1, nl);
    pass(g->de0, de1, nd);
    for (float* x : {g->dtheta, g->dwr, g->dwi})
      if (e == cudaSuccess) e = cudaMemsetAsync(x, 0, (size_t)a->L * sizeof(float), st);
    if (e != cudaSuccess) return cuda_fail(e, "sca2_short_bwd(T=0)");
    return SCA2_OK;
  }
  if (!dO || !g->dkh || !g->dkz || !g->dv || !work) return fail(SCA2_ERR_ARG, "short: null dO, gradient or workspace");
  cudaError_t e = sca2::short_bwd(*a, dO, dc1, ds1, de1, *g, static_cast<float*>(work), max_optin_smem(), st);
  if (e != cudaSuccess) return cuda_fail(e, "sca2_short_bwd");
  return SCA2_OK;
}

}  // extern "C"
