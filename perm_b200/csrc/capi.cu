// extern "C" entry points of libcoldpress_cuda.so (declared in include/coldpress_cuda.h).
// Argument checks and workspace carving live here; the kernels are in the other units.
#include <cuda_runtime.h>
#include <cstdio>
#include <cstring>
#include <vector>
#include "../../include/coldpress_cuda.h"
#include "ef_kernels.h"
#include "kq_common.cuh"
#include "kquant_kernels.h"
#include "xtx_kernels.h"
#include "layout_kernels.h"

static_assert(cpk::kNoAllocScratchBytes == CP_NOALLOC_SCRATCH_BYTES,
              "the public no-allocation limit must equal the scratch array's size");

namespace {

thread_local char g_err[512] = "";
// cp_xtx_inject_stall: armed for the calling thread's next cp_xtx_accumulate only
thread_local int g_xtx_stall_step = -1;
thread_local int64_t g_xtx_stall_wait_ns = 0;

int set_err(int code, const char* msg) {
  std::snprintf(g_err, sizeof(g_err), "%s", msg);
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    std::snprintf(g_err, sizeof(g_err), "%s: %s", what, cudaGetErrorString(e));
    return CP_ERR_CUDA;
  }
  return CP_OK;
}

int check_rc(int rc, const char* what) {
  if (rc == 1) return set_err(CP_ERR_TYPE, what);
  if (rc == 2) return set_err(CP_ERR_SHAPE, what);
  if (rc != 0) return set_err(CP_ERR_ARG, what);
  return check_launch(what);
}

bool is_k_type(int t) { return t == cpk::kQ2_K || t == cpk::kQ3_K || t == cpk::kQ4_K || t == cpk::kQ5_K || t == cpk::kQ6_K; }

int check_shape(int t, int64_t nrow, int64_t n, bool allow_q80) {
  if (!(is_k_type(t) || (allow_q80 && t == cpk::kQ8_0)))
    return set_err(CP_ERR_TYPE, "unsupported ggml type (k-quants Q2_K..Q6_K, and Q8_0 where noted)");
  const int64_t blk = (t == cpk::kQ8_0) ? 32 : 256;
  if (nrow < 0 || n <= 0 || n % blk) return set_err(CP_ERR_SHAPE, "n must be a positive multiple of the block size");
  if (nrow > (int64_t)1 << 31 || n > (int64_t)1 << 30) return set_err(CP_ERR_SHAPE, "tensor too large");
  return CP_OK;
}

size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

// Optional per-kernel-class timing: when enabled, each launch below is bracketed by two CUDA
// events recorded on its stream; cp_profile_collect sums the elapsed times per class.
// Host-thread-local and not thread-safe, like the rest of the calling convention.
enum ProfClass { kProfFit = 0, kProfSweep = 1, kProfFactor = 2, kProfOther = 3, kProfClasses = 4 };
struct ProfMark {
  int cls;
  cudaEvent_t a, b;
};
thread_local bool g_prof = false;
thread_local std::vector<ProfMark> g_marks;
thread_local std::vector<cudaEvent_t> g_free_events;

cudaEvent_t prof_event() {
  if (!g_free_events.empty()) {
    cudaEvent_t e = g_free_events.back();
    g_free_events.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

struct ProfScope {
  bool on;
  ProfMark m;
  cudaStream_t s;
  ProfScope(int cls, cudaStream_t stream) : on(g_prof), s(stream) {
    if (!on) return;
    m.cls = cls;
    m.a = prof_event();
    m.b = prof_event();
    cudaEventRecord(m.a, s);
  }
  ~ProfScope() {
    if (!on) return;
    cudaEventRecord(m.b, s);
    g_marks.push_back(m);
  }
};

struct EfLayout {
  size_t sweep, wcur, dl, ml, codes, total;
};

EfLayout ef_layout(int t, int64_t nrow, int64_t n) {
  int sbw = 16, lo, hi;
  bool hm;
  cpk::grid_spec(t, &sbw, &lo, &hi, &hm);
  EfLayout L;
  size_t off = 0;
  L.sweep = off; off += align256(cpk::ef_sweep_workspace_bytes(nrow, n));
  L.wcur = off; off += align256((size_t)nrow * n * sizeof(float));
  L.dl = off; off += align256((size_t)nrow * (n / sbw) * sizeof(float));
  L.ml = off; off += align256((size_t)nrow * (n / sbw) * sizeof(float));
  L.codes = off; off += align256((size_t)nrow * n);
  L.total = off;
  return L;
}

}  // namespace

extern "C" {

int cp_version(void) { return 100; }

void cp_profile_enable(int on) { g_prof = on != 0; }

int64_t cp_launch_count(void) { return cpk::g_launches.load(); }

int cp_profile_collect(double* ms, int64_t* launches) {
  for (int c = 0; c < kProfClasses; c++) {
    if (ms) ms[c] = 0.0;
    if (launches) launches[c] = 0;
  }
  int rc = CP_OK;
  for (const ProfMark& m : g_marks) {
    float t = 0.0f;
    if (cudaEventSynchronize(m.b) != cudaSuccess || cudaEventElapsedTime(&t, m.a, m.b) != cudaSuccess) {
      rc = check_launch("cp_profile_collect");
    } else {
      if (ms) ms[m.cls] += t;
      if (launches) launches[m.cls] += 1;
    }
    g_free_events.push_back(m.a);
    g_free_events.push_back(m.b);
  }
  g_marks.clear();
  return rc;
}

const char* cp_last_error(void) { return g_err; }

int cp_block_bytes(int ggml_type) { return cpk::block_bytes(ggml_type); }

int cp_kquant_encode(int t, const float* x, int64_t nrow, int64_t n, const float* qw, uint8_t* out, void* stream) {
  if (int rc = check_shape(t, nrow, n, true)) return rc;
  if ((!x || !out) && nrow > 0) return set_err(CP_ERR_ARG, "null pointer");
  if (((uintptr_t)x | (uintptr_t)qw) & 15) return set_err(CP_ERR_ARG, "x and qw must be 16-byte aligned");
  if (t != cpk::kQ8_0 && ((uintptr_t)out & 15)) return set_err(CP_ERR_ARG, "out must be 16-byte aligned");
  ProfScope ps(kProfFit, (cudaStream_t)stream);
  return check_rc(cpk::launch_quantize(t, x, nrow, n, qw, out, (cudaStream_t)stream), "cp_kquant_encode");
}

int cp_kquant_decode(int t, const uint8_t* raw, int64_t nrow, int64_t n, float* out, void* stream) {
  if (int rc = check_shape(t, nrow, n, true)) return rc;
  if ((!raw || !out) && nrow > 0) return set_err(CP_ERR_ARG, "null pointer");
  return check_rc(cpk::launch_dequantize(t, raw, nrow, n, out, (cudaStream_t)stream), "cp_kquant_decode");
}

int cp_grid_params(int t, const uint8_t* raw, int64_t nrow, int64_t n, float* dl, float* ml, void* stream) {
  if (int rc = check_shape(t, nrow, n, false)) return rc;
  if ((!raw || !dl) && nrow > 0) return set_err(CP_ERR_ARG, "null pointer");
  return check_rc(cpk::launch_grid_params(t, raw, nrow, n, dl, ml, (cudaStream_t)stream), "cp_grid_params");
}

int cp_kquant_codes(int t, const uint8_t* raw, int64_t nrow, int64_t n, int8_t* codes, void* stream) {
  if (int rc = check_shape(t, nrow, n, false)) return rc;
  if ((!raw || !codes) && nrow > 0) return set_err(CP_ERR_ARG, "null pointer");
  return check_rc(cpk::launch_codes(t, raw, nrow, n, codes, (cudaStream_t)stream), "cp_kquant_codes");
}

int cp_kquant_repack(int t, uint8_t* raw, const int8_t* codes, int64_t nrow, int64_t n, void* stream) {
  if (int rc = check_shape(t, nrow, n, false)) return rc;
  if ((!raw || !codes) && nrow > 0) return set_err(CP_ERR_ARG, "null pointer");
  return check_rc(cpk::launch_repack(t, raw, codes, nrow, n, (cudaStream_t)stream), "cp_kquant_repack");
}

int cp_weighted_err(int t, const uint8_t* raw, const float* x, const float* w, int64_t nrow, int64_t n, double* out,
                    void* stream) {
  if (int rc = check_shape(t, nrow, n, false)) return rc;
  if (!out || ((!raw || !x) && nrow > 0)) return set_err(CP_ERR_ARG, "null pointer");
  return check_rc(cpk::launch_weighted_err(t, raw, x, w, nrow, n, out, (cudaStream_t)stream), "cp_weighted_err");
}

int cp_hessian_decode(const uint16_t* h16, const float* diag32, double hscale, int64_t d, double* H, void* stream) {
  if (d <= 0 || d > 65536) return set_err(CP_ERR_SHAPE, "d out of range");
  if (!h16 || !H) return set_err(CP_ERR_ARG, "null pointer");
  ProfScope ps(kProfOther, (cudaStream_t)stream);
  return check_rc(cpk::launch_hessian_decode(h16, diag32, hscale, d, H, (cudaStream_t)stream), "cp_hessian_decode");
}

size_t cp_factor_workspace_bytes(int64_t n) { return n > 0 ? cpk::factor_workspace_bytes(n) : 0; }

static int factor_common(const double* H, int64_t n, const int32_t* order, double diag_shift, void* U_out,
                         bool f64, void* workspace, size_t ws_bytes, int32_t* status_dev, void* stream) {
  if (n <= 0 || n % 64) return set_err(CP_ERR_SHAPE, "n must be a positive multiple of 64");
  if (n > 65536) return set_err(CP_ERR_SHAPE, "n too large");
  if (!H || !order || !U_out || !workspace || !status_dev) return set_err(CP_ERR_ARG, "null pointer");
  if (ws_bytes < cpk::factor_workspace_bytes(n)) return set_err(CP_ERR_WORKSPACE, "factor workspace too small");
  ProfScope ps(kProfFactor, (cudaStream_t)stream);
  return check_rc(cpk::launch_factor_u(H, n, order, diag_shift, U_out, f64, workspace, status_dev,
                                       (cudaStream_t)stream),
                  "cp_factor_u");
}

int cp_factor_u(const double* H, int64_t n, const int32_t* order, double diag_shift, float* U_out, void* workspace,
                size_t ws_bytes, int32_t* status_dev, void* stream) {
  return factor_common(H, n, order, diag_shift, U_out, false, workspace, ws_bytes, status_dev, stream);
}

int cp_factor_u_f64(const double* H, int64_t n, const int32_t* order, double diag_shift, double* U_out,
                    void* workspace, size_t ws_bytes, int32_t* status_dev, void* stream) {
  return factor_common(H, n, order, diag_shift, U_out, true, workspace, ws_bytes, status_dev, stream);
}

size_t cp_ef_u_bytes(int64_t n) { return n > 0 ? cpk::ef_u_prepared_bytes(n) : 0; }

int cp_ef_prepare_u(const float* U, int64_t n, float* u_prepared, void* stream) {
  if (n <= 0 || n % 256) return set_err(CP_ERR_SHAPE, "n must be a positive multiple of 256");
  if (!U || !u_prepared) return set_err(CP_ERR_ARG, "null pointer");
  if ((((uintptr_t)U) | ((uintptr_t)u_prepared)) & 15) return set_err(CP_ERR_ARG, "U and u_prepared must be 16-byte aligned");
  return check_rc(cpk::launch_prepare_u(U, n, u_prepared, (cudaStream_t)stream),
                  "cp_ef_prepare_u");
}

size_t cp_ef_sweep_workspace_bytes(int64_t nrow, int64_t n) {
  return (nrow > 0 && n > 0) ? cpk::ef_sweep_workspace_bytes(nrow, n) : 0;
}

int cp_ef_sweep(int t, const float* x, int64_t nrow, int64_t n, const int32_t* order,
                const float* ut2, const float* dl, const float* ml, int8_t* codes, float* w_out, void* workspace,
                size_t ws_bytes, void* stream) {
  if (int rc = check_shape(t, nrow, n, false)) return rc;
  if (nrow == 0) return CP_OK;
  int sbw, lo, hi;
  bool hm;
  cpk::grid_spec(t, &sbw, &lo, &hi, &hm);
  if (!x || !order || !ut2 || !dl || (hm && !ml) || !codes || !workspace) return set_err(CP_ERR_ARG, "null pointer");
  if (ws_bytes < cpk::ef_sweep_workspace_bytes(nrow, n)) return set_err(CP_ERR_WORKSPACE, "sweep workspace too small");
  ProfScope ps(kProfSweep, (cudaStream_t)stream);
  return check_rc(cpk::launch_ef_sweep(t, x, nrow, n, order, ut2, dl, ml, workspace, codes,
                                       w_out, (cudaStream_t)stream),
                  "cp_ef_sweep");
}

int cp_ef_sweep_noalloc(int t, const float* x, int64_t nrow, int64_t n, const int32_t* order, const float* ut2,
                        const float* dl, const float* ml, int8_t* codes, float* w_out, void* stream) {
  if (int rc = check_shape(t, nrow, n, false)) return rc;
  if (nrow == 0) return CP_OK;
  int sbw, lo, hi;
  bool hm;
  cpk::grid_spec(t, &sbw, &lo, &hi, &hm);
  if (!x || !order || !ut2 || !dl || (hm && !ml) || !codes) return set_err(CP_ERR_ARG, "null pointer");
  if (cpk::ef_sweep_workspace_bytes(nrow, n) > cpk::kNoAllocScratchBytes) {
    const int pad = 32 * cpk::kSweepWarps;
    std::snprintf(g_err, sizeof(g_err),
                  "cp_ef_sweep_noalloc: ceil(nrow/%d)*%d * n * 4 bytes = %zu exceeds the fixed %zu-byte scratch; "
                  "use cp_ef_sweep with a workspace",
                  pad, pad, cpk::ef_sweep_workspace_bytes(nrow, n), cpk::kNoAllocScratchBytes);
    return CP_ERR_WORKSPACE;
  }
  const int rc = cpk::launch_ef_sweep_noalloc(t, x, nrow, n, order, ut2, dl, ml, codes, w_out, (cudaStream_t)stream);
  if (rc == 4) {
    // a failed CUDA call leaves its error pending; a lookup that "succeeded" with a null
    // address leaves none, and must not be reported as a sweep that ran
    if (check_launch("cp_ef_sweep_noalloc: locating the fixed scratch") == CP_OK)
      return set_err(CP_ERR_CUDA, "cp_ef_sweep_noalloc: the fixed scratch has no device address on this device");
    return CP_ERR_CUDA;
  }
  if (rc == 5) return set_err(CP_ERR_ARG, "cp_ef_sweep_noalloc: device index out of range");
  return check_rc(rc, "cp_ef_sweep_noalloc");
}

size_t cp_ef_workspace_bytes(int t, int64_t nrow, int64_t n) {
  if (!is_k_type(t) || nrow <= 0 || n <= 0) return 0;
  return ef_layout(t, nrow, n).total;
}

int cp_ef_encode(int t, const float* x, int64_t nrow, int64_t n, const int32_t* order, const float* ut2, const float* qw,
                 int n_iter, uint8_t* out, uint8_t* first_fit_out, void* workspace, size_t ws_bytes, void* stream) {
  if (int rc = check_shape(t, nrow, n, false)) return rc;
  if (nrow == 0) return CP_OK;
  if (n_iter < 1 || n_iter > 64) return set_err(CP_ERR_ARG, "n_iter must be in 1..64");
  if (!x || !order || !ut2 || !out || !workspace) return set_err(CP_ERR_ARG, "null pointer");
  if (((uintptr_t)x | (uintptr_t)qw | (uintptr_t)out | (uintptr_t)workspace) & 15)
    return set_err(CP_ERR_ARG, "x, qw, out and workspace must be 16-byte aligned");
  const EfLayout L = ef_layout(t, nrow, n);
  if (ws_bytes < L.total) return set_err(CP_ERR_WORKSPACE, "ef workspace too small");
  cudaStream_t s = (cudaStream_t)stream;
  char* ws = (char*)workspace;
  float* wcur = (float*)(ws + L.wcur);
  float* dl = (float*)(ws + L.dl);
  float* ml = (float*)(ws + L.ml);
  int8_t* codes = (int8_t*)(ws + L.codes);
  int rc;
  for (int it = 0; it < n_iter; it++) {
    // commit the grid from the current (compensated) weights; round 1 starts from x
    const float* src = it == 0 ? x : wcur;
    {
      ProfScope ps(kProfFit, s);
      if ((rc = check_rc(cpk::launch_quantize(t, src, nrow, n, qw, out, s), "cp_ef_encode: fit"))) return rc;
    }
    if (it == 0 && first_fit_out) {
      const size_t nb = (size_t)nrow * (n / 256) * cpk::block_bytes(t);
      if (cudaMemcpyAsync(first_fit_out, out, nb, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
        return check_launch("cp_ef_encode: first-fit copy");
    }
    if ((rc = check_rc(cpk::launch_grid_params(t, out, nrow, n, dl, ml, s), "cp_ef_encode: grid"))) return rc;
    {
      ProfScope ps(kProfSweep, s);
      if ((rc = check_rc(cpk::launch_ef_sweep(t, x, nrow, n, order, ut2, dl, ml, ws + L.sweep,
                                              codes, it + 1 < n_iter ? wcur : nullptr, s),
                         "cp_ef_encode: sweep")))
        return rc;
    }
    if ((rc = check_rc(cpk::launch_repack(t, out, codes, nrow, n, s), "cp_ef_encode: repack"))) return rc;
  }
  return CP_OK;
}

// ---------------------------------------------------------------------------- grouped calls

int cp_kquant_encode_batch(int t, const cp_fit_job* jobs, int count, void* stream) {
  if (count < 0 || (count > 0 && !jobs)) return set_err(CP_ERR_ARG, "bad job list");
  if (!is_k_type(t)) return set_err(CP_ERR_TYPE, "grouped fits support the k-quant types");
  cudaStream_t s = (cudaStream_t)stream;
  for (int pass = 0; pass < 2; pass++) {  // imatrix jobs, then reference-path jobs
    static thread_local cpk::FitBatch b;
    b.count = 0;
    int64_t ctas = 0;
    for (int i = 0; i <= count; i++) {
      const bool flush = (i == count) || b.count == cpk::kFitBatchMax;
      if (flush && b.count) {
        ProfScope ps(kProfFit, s);
        if (int rc = check_rc(cpk::launch_quantize_batch(t, pass == 0, b, ctas, s), "cp_kquant_encode_batch")) return rc;
        b.count = 0;
        ctas = 0;
      }
      if (i == count) break;
      const cp_fit_job& j = jobs[i];
      if ((j.qw != nullptr) != (pass == 0)) continue;
      if (int rc = check_shape(t, j.nrow, j.n, false)) return rc;
      if (j.nrow == 0) continue;
      if (!j.x || !j.out || (((uintptr_t)j.x | (uintptr_t)j.qw | (uintptr_t)j.out) & 15))
        return set_err(CP_ERR_ARG, "null or unaligned pointer in a fit job");
      cpk::FitDesc& d = b.d[b.count++];
      d.x = j.x;
      d.qw = j.qw;
      d.out = j.out;
      d.nsb_row = j.n / 256;
      d.nsb = j.nrow * d.nsb_row;
      d.cta0 = ctas;
      ctas += cpk::quantize_batch_ctas(t, d.nsb);
    }
  }
  return CP_OK;
}

static int block_batch(int op, const cp_block_job* jobs, int count, void* stream, const char* what) {
  if (count < 0 || (count > 0 && !jobs)) return set_err(CP_ERR_ARG, "bad job list");
  cudaStream_t s = (cudaStream_t)stream;
  static thread_local cpk::SbBatch b;
  b.count = 0;
  int64_t total = 0;
  for (int i = 0; i <= count; i++) {
    const bool flush = (i == count) || b.count == cpk::kSbBatchMax;
    if (flush && b.count) {
      ProfScope ps(kProfOther, s);
      if (int rc = check_rc(cpk::launch_sb_batch(op, b, total, s), what)) return rc;
      b.count = 0;
      total = 0;
    }
    if (i == count) break;
    const cp_block_job& j = jobs[i];
    if (int rc = check_shape(j.ggml_type, j.nrow, j.n, false)) return rc;
    if (j.nrow == 0) continue;
    const bool ok = op == 0 ? (j.raw && j.dl) : op == 1 ? (j.raw_out && j.codes) : (j.raw && j.x && j.err);
    if (!ok) return set_err(CP_ERR_ARG, "null pointer in a block job");
    if (op == 0 && j.grid_pitch != 0 && j.grid_pitch < j.nrow) return set_err(CP_ERR_ARG, "grid_pitch < nrow");
    if (op == 1 && (((uintptr_t)j.codes) & 15)) return set_err(CP_ERR_ARG, "codes must be 16-byte aligned");
    cpk::SbDesc& d = b.d[b.count++];
    d.raw = j.raw;
    d.raw_w = j.raw_out;
    d.codes = j.codes;
    d.x = j.x;
    d.w = j.w;
    d.dl = j.dl;
    d.ml = j.ml;
    d.err = j.err;
    d.nsb_row = j.n / 256;
    d.nsb = j.nrow * d.nsb_row;
    d.sb0 = total;
    d.gpitch = op == 0 ? j.grid_pitch : 0;
    d.type = j.ggml_type;
    total += (d.nsb + 15) / 16;   // 16 superblocks per CTA
  }
  return CP_OK;
}

int cp_grid_params_batch(const cp_block_job* jobs, int count, void* stream) {
  return block_batch(0, jobs, count, stream, "cp_grid_params_batch");
}

int cp_kquant_repack_batch(const cp_block_job* jobs, int count, void* stream) {
  return block_batch(1, jobs, count, stream, "cp_kquant_repack_batch");
}

int cp_weighted_err_batch(const cp_block_job* jobs, int count, void* stream) {
  return block_batch(2, jobs, count, stream, "cp_weighted_err_batch");
}

int cp_ef_sweep_batch(const cp_sweep_job* jobs, int count, void* stream) {
  if (count < 0 || (count > 0 && !jobs)) return set_err(CP_ERR_ARG, "bad job list");
  cudaStream_t s = (cudaStream_t)stream;
  static thread_local cpk::SweepBatch b;
  // A launch too small to keep the GPU busy is bounded by its longest rows, whose columns one
  // lane walks serially; such a launch runs the column-split form, several warps per 32 rows,
  // each applying the errors to its share of every block: four warps under one and a half
  // waves of four resident 128-row CTAs per SM, two under two waves (measured crossovers).
  const int sms = cpk::device_sm_count();
  int64_t plain = 0;
  for (int i = 0; i < count; i++)
    if (jobs[i].nrow > 0) plain += cpk::sweep_ctas(jobs[i].nrow);
  const int split = plain < 6LL * sms ? 4 : plain < 8LL * sms ? 2 : 1;
  b.count = 0;
  int tiles = 0;
  for (int i = 0; i <= count; i++) {
    const bool flush = (i == count) || b.count == cpk::kSweepBatchMax;
    if (flush && b.count) {
      ProfScope ps(kProfSweep, s);
      if (int rc = check_rc(cpk::launch_ef_sweep_batch(b, tiles, split, s), "cp_ef_sweep_batch"))
        return rc;
      b.count = 0;
      tiles = 0;
    }
    if (i == count) break;
    const cp_sweep_job& j = jobs[i];
    if (int rc = check_shape(j.ggml_type, j.nrow, j.n, false)) return rc;
    if (j.nrow == 0) continue;
    if (!j.x || !j.order || !j.u_prepared || !j.dl || !j.codes || !j.workspace)
      return set_err(CP_ERR_ARG, "null pointer in a sweep job");
    cpk::SweepDesc& d = b.d[b.count];
    if (!cpk::sweep_desc(j.ggml_type, j.x, j.nrow, j.n, j.order, j.u_prepared, j.dl, j.ml, j.workspace, j.codes,
                         j.w_out, &d))
      return set_err(CP_ERR_TYPE, "cp_ef_sweep_batch: unsupported type");
    if (d.ml == nullptr && (j.ggml_type == cpk::kQ2_K || j.ggml_type == cpk::kQ4_K || j.ggml_type == cpk::kQ5_K))
      return set_err(CP_ERR_ARG, "ml is required for Q2_K/Q4_K/Q5_K");
    if (j.pitch != 0 && j.pitch < cpk::sweep_rows_padded(j.nrow))
      return set_err(CP_ERR_ARG, "cp_ef_sweep_batch: pitch < cp_ef_sweep_rows(nrow)");
    if (j.pitch > (int64_t)1 << 31) return set_err(CP_ERR_SHAPE, "cp_ef_sweep_batch: pitch too large");
    d.pitch = (int)j.pitch;
    d.tile0 = tiles;
    tiles += split > 1 ? cpk::sweep_split_ctas(j.nrow, split) : cpk::sweep_ctas(j.nrow);
    b.count++;
  }
  return CP_OK;
}

int64_t cp_ef_sweep_rows(int64_t nrow) { return nrow > 0 ? cpk::sweep_rows_padded(nrow) : 0; }

int cp_transpose_batch(const cp_transpose_job* jobs, int count, void* stream) {
  if (count < 0 || (count > 0 && !jobs)) return set_err(CP_ERR_ARG, "bad job list");
  cudaStream_t s = (cudaStream_t)stream;
  static thread_local cpk::TrBatch b;
  for (int eb : {4, 1}) {
    b.count = 0;
    int64_t tiles = 0;
    for (int i = 0; i <= count; i++) {
      const bool flush = (i == count) || b.count == cpk::kTrBatchMax;
      if (flush && b.count) {
        ProfScope ps(kProfOther, s);
        if (int rc = check_rc(cpk::launch_transpose_batch(b, eb, tiles, s), "cp_transpose_batch")) return rc;
        b.count = 0;
        tiles = 0;
      }
      if (i == count) break;
      const cp_transpose_job& j = jobs[i];
      if (j.elem_bytes != 1 && j.elem_bytes != 4) return set_err(CP_ERR_ARG, "elem_bytes must be 1 or 4");
      if (j.elem_bytes != eb || j.rows == 0 || j.cols == 0) continue;
      if (j.rows < 0 || j.cols < 0 || j.src_ld < j.cols || j.dst_ld < j.rows)
        return set_err(CP_ERR_SHAPE, "cp_transpose_batch: bad rows, cols or leading dimensions");
      if (!j.src || !j.dst) return set_err(CP_ERR_ARG, "null pointer in a transpose job");
      cpk::TrDesc& d = b.d[b.count++];
      d.src = j.src;
      d.dst = j.dst;
      d.rows = j.rows;
      d.cols = j.cols;
      d.src_ld = j.src_ld;
      d.dst_ld = j.dst_ld;
      const int T = cpk::transpose_tile_dim(eb);
      d.tiles_c = (j.cols + T - 1) / T;
      d.tile0 = tiles;
      tiles += cpk::transpose_tiles(j.rows, j.cols, eb);
    }
  }
  return CP_OK;
}

int cp_fetch_host(void* dst, const void* src_host, int64_t bytes, void* stream) {
  if (bytes < 0) return set_err(CP_ERR_SHAPE, "cp_fetch_host: negative size");
  if (bytes == 0) return CP_OK;
  if (!dst || !src_host) return set_err(CP_ERR_ARG, "null pointer");
  void* mapped = nullptr;
  if (cudaHostGetDevicePointer(&mapped, const_cast<void*>(src_host), 0) != cudaSuccess || !mapped) {
    cudaGetLastError();
    return set_err(CP_ERR_ARG, "cp_fetch_host: the source is not pinned (mapped) host memory");
  }
  ProfScope ps(kProfOther, (cudaStream_t)stream);
  return check_rc(cpk::launch_fetch_host(dst, mapped, bytes, (cudaStream_t)stream), "cp_fetch_host");
}

int cp_gather_f32(const float* x, int64_t ld, const int64_t* rows, int64_t nrow_out, const int64_t* cols,
                  int64_t n_out, float* out, void* stream) {
  if (nrow_out < 0 || n_out < 0 || ld < 0) return set_err(CP_ERR_SHAPE, "cp_gather_f32: negative size");
  if (nrow_out == 0 || n_out == 0) return CP_OK;
  if (!x || !out) return set_err(CP_ERR_ARG, "null pointer");
  if (!cols && ld < n_out) return set_err(CP_ERR_SHAPE, "cp_gather_f32: ld smaller than the row");
  ProfScope ps(kProfOther, (cudaStream_t)stream);
  return check_rc(cpk::launch_gather_f32(x, ld, rows, nrow_out, cols, n_out, out, (cudaStream_t)stream),
                  "cp_gather_f32");
}

int cp_col_sqdiff(const float* x, const float* y, int64_t nrow, int64_t n, int64_t ld, double* out, void* stream) {
  if (nrow < 0 || n < 0 || ld < n) return set_err(CP_ERR_SHAPE, "cp_col_sqdiff: bad nrow, n or ld");
  if (n == 0) return CP_OK;
  if (!x || !out) return set_err(CP_ERR_ARG, "null pointer");
  ProfScope ps(kProfOther, (cudaStream_t)stream);
  return check_rc(cpk::launch_col_sqdiff(x, y, nrow, n, ld, out, (cudaStream_t)stream), "cp_col_sqdiff");
}

int cp_factor_u_batch(const cp_factor_job* jobs, int count, void* stream) {
  if (count < 0 || (count > 0 && !jobs)) return set_err(CP_ERR_ARG, "bad job list");
  cudaStream_t s = (cudaStream_t)stream;
  std::vector<int> done(count, 0);
  static thread_local cpk::FactorBatch fb;
  for (int i = 0; i < count; i++) {
    const cp_factor_job& j = jobs[i];
    if (j.n <= 0 || j.n % 64 || j.n > 65536) return set_err(CP_ERR_SHAPE, "n must be a positive multiple of 64");
    if (!j.H || !j.order || !j.U_out || !j.workspace || !j.status_dev) return set_err(CP_ERR_ARG, "null pointer");
    if (((uintptr_t)j.workspace) & 15) return set_err(CP_ERR_ARG, "workspace must be 16-byte aligned");
  }
  for (int i = 0; i < count; i++) {
    if (done[i]) continue;
    fb.count = 0;
    fb.n = (int)jobs[i].n;
    fb.out_f64 = 0;
    for (int k = i; k < count && fb.count < cpk::kFactorBatchMax; k++) {
      if (done[k] || jobs[k].n != jobs[i].n) continue;
      const int b = fb.count++;
      fb.H[b] = jobs[k].H;
      fb.order[b] = jobs[k].order;
      fb.P[b] = (double*)jobs[k].workspace;
      fb.U[b] = jobs[k].U_out;
      fb.status[b] = jobs[k].status_dev;
      fb.shift[b] = jobs[k].diag_shift;
      done[k] = 1;
    }
    ProfScope ps(kProfFactor, s);
    if (int rc = check_rc(cpk::launch_factor_batch(fb, s), "cp_factor_u_batch")) return rc;
    i--;  // revisit: there may be more jobs of this size than one batch holds
  }
  return CP_OK;
}


size_t cp_xtx_workspace_bytes(int dtype, int64_t T, int64_t d) {
  if (T < 0 || d <= 0 || (dtype != CP_XTX_BF16 && dtype != CP_XTX_F32)) return 0;
  return cpk::xtx_plan(T, d, dtype == CP_XTX_F32, cpk::device_sm_count()).ws_bytes;
}

int cp_xtx_accumulate(int dtype, const void* x, int64_t T, int64_t d, float* H, void* workspace, size_t ws_bytes,
                      void* stream) {
  if (dtype != CP_XTX_BF16 && dtype != CP_XTX_F32) return set_err(CP_ERR_TYPE, "dtype must be CP_XTX_BF16 or CP_XTX_F32");
  if (T < 0 || d <= 0 || d % 8) return set_err(CP_ERR_SHAPE, "d must be a positive multiple of 8");
  if (d > (1 << 30) || T > (int64_t)1 << 30) return set_err(CP_ERR_SHAPE, "T or d too large");
  if (T == 0) return CP_OK;
  if (!x || !H || !workspace) return set_err(CP_ERR_ARG, "null pointer");
  if (((uintptr_t)x | (uintptr_t)H | (uintptr_t)workspace) & 15)
    return set_err(CP_ERR_ARG, "x, H and workspace must be 16-byte aligned");
  const cpk::XtxPlan p = cpk::xtx_plan(T, d, dtype == CP_XTX_F32, cpk::device_sm_count());
  if (ws_bytes < p.ws_bytes) return set_err(CP_ERR_WORKSPACE, "workspace smaller than cp_xtx_workspace_bytes()");
  cudaStream_t s = (cudaStream_t)stream;
  ProfScope ps(kProfOther, s);
  const int skip = g_xtx_stall_step;
  const unsigned long long wait_ns = (unsigned long long)g_xtx_stall_wait_ns;
  g_xtx_stall_step = -1;   // one-shot
  g_xtx_stall_wait_ns = 0;
  const int rc = cpk::launch_xtx(x, dtype == CP_XTX_F32, T, d, H, workspace, p, s, skip, wait_ns);
  if (rc == 1) return set_err(CP_ERR_CUDA, "cp_xtx_accumulate: kernel attribute or memset failed");
  if (rc == 2) return set_err(CP_ERR_CUDA, "cp_xtx_accumulate: cuTensorMapEncodeTiled unavailable from the driver");
  if (rc == 3) return set_err(CP_ERR_CUDA, "cp_xtx_accumulate: cuTensorMapEncodeTiled rejected the activation layout");
  return check_launch("cp_xtx_accumulate");
}

int cp_xtx_inject_stall(int skip_step, int64_t wait_ns) {
  if (skip_step < 0 || wait_ns < 1000 || wait_ns > 2000000000LL)
    return set_err(CP_ERR_ARG, "cp_xtx_inject_stall: skip_step >= 0 and 1 us <= wait_ns <= 2 s");
  g_xtx_stall_step = skip_step;
  g_xtx_stall_wait_ns = wait_ns;
  return CP_OK;
}

int cp_xtx_status(void* workspace, void* stream) {
  if (!workspace) return set_err(CP_ERR_ARG, "null pointer");
  int st = 0;
  cudaStream_t s = (cudaStream_t)stream;
  if (cudaMemcpyAsync(&st, workspace, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return check_launch("cp_xtx_status");
  if (st == 0) return CP_OK;
  if (cudaMemsetAsync(workspace, 0, 4, s) != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess)
    return check_launch("cp_xtx_status");
  return set_err(CP_ERR_TIMEOUT, "a bounded wait in cp_xtx_accumulate ran out; H is incomplete");
}

}  // extern "C"
