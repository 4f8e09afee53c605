// C ABI of the gmdn B200 scan library (declared in include/gmdn_scan.h).
//
// Validates arguments, carves the caller's workspace / saved buffers and
// enqueues the kernels on the caller's stream.  Nothing is allocated and
// nothing synchronises the host.

#include <atomic>
#include <initializer_list>
#include <cstdarg>
#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/gmdn_scan.h"
#include "scan_kernels.h"
#include "fast_path.h"

namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(GMDN_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
}

constexpr size_t kAlign = 256;
inline size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// Sequential carving of a caller buffer into 256-byte aligned pieces.
struct Carver {
  char* base;
  size_t used = 0;
  explicit Carver(void* p) : base(static_cast<char*>(p)) {}
  float* take(size_t n_floats) {
    float* p = base ? reinterpret_cast<float*>(base + used) : nullptr;
    used += align_up(n_floats * sizeof(float));
    return p;
  }
};

bool dh_ok(int dh) { return dh == 16 || dh == 32 || dh == 64 || dh == 128; }

int check_common(int B, int H, int N, int dh, int rule, int ns, int precision) {
  if (B < 0 || H < 0 || N < 0) return fail(GMDN_ERR_INVALID, "negative size B=%d H=%d N=%d", B, H, N);
  if (rule < 0 || rule > 2) return fail(GMDN_ERR_INVALID, "rule must be 0, 1 or 2 (got %d)", rule);
  if (ns < 0 || ns > 16) return fail(GMDN_ERR_INVALID, "ns must be in [0, 16] (got %d)", ns);
  if (precision != GMDN_PREC_IEEE && precision != GMDN_PREC_FAST)
    return fail(GMDN_ERR_INVALID, "precision must be 0 (ieee) or 1 (fast) (got %d)", precision);
  if (!dh_ok(dh))
    return fail(GMDN_ERR_UNSUPPORTED, "head dim %d not built (16, 32, 64, 128)", dh);
  return GMDN_OK;
}

size_t mats(size_t count, int dh) { return count * static_cast<size_t>(dh) * dh; }

size_t scan_scratch_floats(int BH, int dh, int ns) {
  const int per = gmdn::scan_bwd_scratch_mats(ns) > gmdn::kScanFwdScratchMats
                      ? gmdn::scan_bwd_scratch_mats(ns)
                      : gmdn::kScanFwdScratchMats;
  return mats(static_cast<size_t>(BH) * per, dh);
}

struct ScanSaved {
  float *M_hist, *V_hist;
  size_t bytes;
};

ScanSaved carve_scan_saved(void* saved, int BH, int N, int dh, int rule) {
  Carver c(saved);
  ScanSaved s{nullptr, nullptr, 0};
  const size_t per = mats(static_cast<size_t>(BH) * N, dh);
  if (rule != 0) s.M_hist = c.take(per);
  if (rule == 2) s.V_hist = c.take(per);
  s.bytes = c.used;
  return s;
}

struct ChunkBufs {
  // saved (forward -> backward)
  float *S, *M_hist, *V_hist;   // exact path: fp32 states and moments
  gmdn::TcBufs tc;              // tensor-core path
  size_t saved_bytes;
  // workspace
  uint32_t* status;             // device status word (first 256 bytes)
  float *Kw, *Uv, *gS, *dUv, *dKw;
  float *a_c, *b_c, *m_c, *n_c, *da_c, *db_c, *dm_c, *dn_c;
  float* scratch;
  size_t ws_bytes;
};

// `fast`: the tensor-core path (fused forward, two-kernel backward).  Its
// saved buffer holds the bf16 states S_j (adam: also G_j and the pre-update
// moments); its workspace the device status word, the bf16 cotangents of G_j
// and, for adam, the fp32 moment slabs and the chunk-scalar cotangents.
ChunkBufs carve_chunk(void* saved, void* ws, int BH, int N, int dh, int rule, int ns,
                      bool fast) {
  ChunkBufs b{};
  const size_t sc = static_cast<size_t>(BH) * N;
  Carver cs(saved);
  Carver cw(ws);
  b.status = reinterpret_cast<uint32_t*>(cw.take(64));
  if (fast) {
    // the tensor-core kernels keep every state as 128 x 128 (a dh-64 head is
    // the leading 64 x 64 block, the rest zero)
    dh = 128;
    const size_t per = mats(static_cast<size_t>(BH) * N, dh);
    auto half_mats = [&](Carver& c) { return reinterpret_cast<uint16_t*>(c.take((per + 1) / 2)); };
    b.tc.status = b.status;
    b.tc.S_hist = half_mats(cs);
    if (rule == 2) {
      b.tc.G_hist = half_mats(cs);
      b.tc.Mp_hist = half_mats(cs);
      b.tc.Vp_hist = half_mats(cs);
    }
    if (rule == 1) {
      b.tc.S_lo_hist = half_mats(cs);
      b.tc.M_hist = cs.take(per);
      b.tc.X_hist = reinterpret_cast<uint8_t*>(cs.take(per * static_cast<size_t>(ns)));
    }
    b.saved_bytes = cs.used;
    b.tc.Gbar_hist = half_mats(cw);
    if (rule == 1) b.tc.Gbar_lo_hist = half_mats(cw);
    if (rule == 0) b.tc.progress = reinterpret_cast<uint32_t*>(cw.take(BH));
    if (rule != 0) {
      b.tc.M_ws = cw.take(mats(BH, dh));
      if (rule == 2) b.tc.V_ws = cw.take(mats(BH, dh));
      b.tc.dac = cw.take(sc);
      b.tc.dbc = cw.take(sc);
      b.tc.dmc = cw.take(sc);
      b.tc.dnc = cw.take(sc);
    }
    b.ws_bytes = cw.used;
    return b;
  }
  const size_t per = mats(static_cast<size_t>(BH) * N, dh);
  b.S = cs.take(per);
  b.M_hist = rule != 0 ? cs.take(per) : nullptr;
  b.V_hist = rule == 2 ? cs.take(per) : nullptr;
  b.saved_bytes = cs.used;
  b.Kw = cw.take(per);
  b.Uv = cw.take(per);
  b.gS = cw.take(per);
  b.dUv = cw.take(per);
  b.dKw = cw.take(per);
  b.a_c = cw.take(sc);
  b.b_c = cw.take(sc);
  b.m_c = cw.take(sc);
  b.n_c = cw.take(sc);
  b.da_c = cw.take(sc);
  b.db_c = cw.take(sc);
  b.dm_c = cw.take(sc);
  b.dn_c = cw.take(sc);
  b.scratch = cw.take(scan_scratch_floats(BH, dh, ns));
  b.ws_bytes = cw.used;
  return b;
}

// Shape test for the fused forward, mirroring chunk_fwd_tc_supported().
bool chunk_fast(int dh, int chunk, int rule, int precision, int io_f32, int N) {
  if (precision != GMDN_PREC_FAST || io_f32) return false;
  gmdn::ChunkArgs p{};
  p.dh = dh; p.C = chunk; p.rule = rule; p.io_f32 = false; p.N = N;
  return gmdn::chunk_fwd_tc_supported(p) || gmdn::chunk_fwd_muon_tc_supported(p);
}

int check_chunk(int B, int H, int T, int dh, int chunk, int rule, int ns, int precision) {
  int rc = check_common(B, H, T, dh, rule, ns, precision);
  if (rc) return rc;
  if (chunk != 32 && chunk != 64)
    return fail(GMDN_ERR_UNSUPPORTED, "chunk %d not built (32, 64)", chunk);
  if (T % chunk)
    return fail(GMDN_ERR_INVALID, "seq_len %d must be a multiple of chunk %d", T, chunk);
  return GMDN_OK;
}

// Optional per-launch timing: when enabled, every kernel launch is bracketed
// by two CUDA events on the launching stream; gmdn_prof_report() waits for
// them and returns per-kernel totals.  Off by default (no events recorded).
struct ProfRec {
  const char* name;
  cudaEvent_t start, stop;
};
std::mutex g_prof_mu;
std::atomic<int> g_prof_on{0};
std::vector<ProfRec> g_prof_recs;
std::vector<cudaEvent_t> g_prof_pool;
std::string g_prof_json;

cudaEvent_t prof_event() {
  if (!g_prof_pool.empty()) {
    cudaEvent_t e = g_prof_pool.back();
    g_prof_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

struct ProfScope {
  cudaStream_t st;
  const char* name;
  cudaEvent_t a = nullptr, b = nullptr;
  ProfScope(cudaStream_t s, const char* n) : st(s), name(n) {
    if (g_prof_on.load(std::memory_order_relaxed)) {
      std::lock_guard<std::mutex> lk(g_prof_mu);
      a = prof_event();
      b = prof_event();
      cudaEventRecord(a, st);
    }
  }
  void done() {
    if (a) {
      cudaEventRecord(b, st);
      std::lock_guard<std::mutex> lk(g_prof_mu);
      g_prof_recs.push_back({name, a, b});
    }
  }
};

#define GMDN_LAUNCH(call, what)                            \
  do {                                                     \
    ProfScope ps_(st, what);                               \
    cudaError_t e_ = (call);                               \
    if (e_ != cudaSuccess) return cuda_fail(e_, what);     \
    ps_.done();                                            \
    g_launches.fetch_add(1, std::memory_order_relaxed);    \
  } while (0)

}  // namespace

extern "C" {

int gmdn_abi_version(void) { return 1; }

const char* gmdn_last_error_string(void) { return g_last_error.c_str(); }

uint64_t gmdn_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

int gmdn_chunk_bwd_fused_tiles(int B, int H, int T, int dh, int chunk, int rule, int precision,
                               int io_f32) {
  g_last_error.clear();
  if (B <= 0 || H <= 0 || chunk <= 0 || T <= 0 || T % chunk) return 0;
  const int N = T / chunk;
  if (!chunk_fast(dh, chunk, rule, precision, io_f32, N)) return 0;
  gmdn::ChunkArgs p{};
  p.BH = B * H;
  p.T = T;
  p.N = N;
  p.C = chunk;
  p.dh = dh;
  p.rule = rule;
  p.io_f32 = io_f32 != 0;
  return gmdn::chunk_bwd_fused_tiles(p);
}

int gmdn_selftest_wait_timeout(uint32_t* status, uint64_t limit_ns, void* stream) {
  g_last_error.clear();
  if (!status) return fail(GMDN_ERR_INVALID, "null status pointer");
  const uint64_t lim = limit_ns < 1000000ull ? 1000000ull
                                             : (limit_ns > 2000000000ull ? 2000000000ull : limit_ns);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GMDN_LAUNCH(gmdn::wait_timeout_selftest(status, lim, st), "wait_timeout_selftest");
  return GMDN_OK;
}

static int check_prologue(std::initializer_list<const void*> ptrs, int B, int T, int H, int dh,
                          int n_gates) {
  for (const void* p : ptrs) {
    if (!p) return fail(GMDN_ERR_INVALID, "mixer_prologue: null pointer");
    if (reinterpret_cast<uintptr_t>(p) % 16)
      return fail(GMDN_ERR_INVALID, "mixer_prologue: pointers must be 16-byte aligned");
  }
  if (B < 0 || T < 0 || H < 0) return fail(GMDN_ERR_INVALID, "negative size B=%d T=%d H=%d", B, T, H);
  if (dh != 32 && dh != 64 && dh != 128)
    return fail(GMDN_ERR_UNSUPPORTED, "mixer_prologue: dh must be 32, 64 or 128 (got %d)", dh);
  if (n_gates != 3 && n_gates != 4)
    return fail(GMDN_ERR_INVALID, "mixer_prologue: n_gates must be 3 or 4 (got %d)", n_gates);
  if (static_cast<long long>(B) * T * 3 * H * dh >= (1ll << 31))
    return fail(GMDN_ERR_UNSUPPORTED, "mixer_prologue: B*T*3D must be below 2^31");
  return GMDN_OK;
}

int gmdn_mixer_prologue_fwd(const void* u, const float* conv_w, const float* conv_b,
                            const void* gl, void* q, void* k, void* v, void* g, int B, int T,
                            int H, int dh, int n_gates, int io_f32, void* stream) {
  g_last_error.clear();
  int rc = check_prologue({u, conv_w, conv_b, gl, q, k, v, g}, B, T, H, dh, n_gates);
  if (rc) return rc;
  if (static_cast<long long>(B) * T * H == 0) return GMDN_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GMDN_LAUNCH(gmdn::mixer_prologue_fwd(u, conv_w, conv_b, gl, q, k, v, g, B, T, H, dh, n_gates,
                                       io_f32 != 0, st),
              "mixer_prologue_fwd");
  return GMDN_OK;
}

int gmdn_mixer_prologue_bwd(const void* u, const float* conv_w, const float* conv_b,
                            const void* gl, const void* dq, const void* dk, const void* dv,
                            const void* dg, void* du, float* dconv_w, float* dconv_b, void* dgl,
                            int B, int T, int H, int dh, int n_gates, int io_f32, void* stream) {
  g_last_error.clear();
  int rc = check_prologue({u, conv_w, conv_b, gl, dq, dk, dv, dg, du, dconv_w, dconv_b, dgl}, B, T,
                          H, dh, n_gates);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (static_cast<long long>(B) * T * H == 0) {
    cudaError_t ce = cudaMemsetAsync(dconv_w, 0, sizeof(float) * 3 * H * dh * 4, st);
    if (ce == cudaSuccess) ce = cudaMemsetAsync(dconv_b, 0, sizeof(float) * 3 * H * dh, st);
    return ce == cudaSuccess ? GMDN_OK : cuda_fail(ce, "mixer_prologue_bwd");
  }
  GMDN_LAUNCH(gmdn::mixer_prologue_bwd(u, conv_w, conv_b, gl, dq, dk, dv, dg, du, dconv_w, dconv_b,
                                       dgl, B, T, H, dh, n_gates, io_f32 != 0, st),
              "mixer_prologue_bwd");
  return GMDN_OK;
}

static int check_rmsnorm(const void* o, const float* weight, const void* out, int B, int H,
                         int T, int dh) {
  if (!o || !weight || !out) return fail(GMDN_ERR_INVALID, "null pointer");
  if (B < 0 || H < 0 || T < 0) return fail(GMDN_ERR_INVALID, "negative size B=%d H=%d T=%d", B, H, T);
  if (static_cast<long long>(B) * H * T >= (1ll << 31))
    return fail(GMDN_ERR_UNSUPPORTED, "head_rmsnorm: B*H*T must be below 2^31");
  if (dh != 32 && dh != 64 && dh != 128)
    return fail(GMDN_ERR_UNSUPPORTED, "head_rmsnorm: dh must be 32, 64 or 128 (got %d)", dh);
  for (const void* p : {static_cast<const void*>(o), static_cast<const void*>(weight), out})
    if (reinterpret_cast<uintptr_t>(p) % 16)
      return fail(GMDN_ERR_INVALID, "head_rmsnorm: pointers must be 16-byte aligned");
  return GMDN_OK;
}

int gmdn_head_rmsnorm_fwd(const void* o, const float* weight, void* y, int B, int H, int T,
                          int dh, float eps, int in_f32, int out_f32, void* stream) {
  g_last_error.clear();
  int rc = check_rmsnorm(o, weight, y, B, H, T, dh);
  if (rc) return rc;
  if (static_cast<long long>(B) * H * T == 0) return GMDN_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float e = eps < 0.f ? 1.1920928955078125e-07f : eps;
  GMDN_LAUNCH(gmdn::head_rmsnorm_fwd(o, weight, y, B, H, T, dh, e, in_f32 != 0, out_f32 != 0, st),
              "head_rmsnorm_fwd");
  return GMDN_OK;
}

int gmdn_head_rmsnorm_bwd(const void* o, const float* weight, const void* dy, void* d_o,
                          float* dweight, int B, int H, int T, int dh, float eps, int in_f32,
                          int out_f32, void* stream) {
  g_last_error.clear();
  int rc = check_rmsnorm(o, weight, d_o, B, H, T, dh);
  if (rc) return rc;
  if (!dy || !dweight) return fail(GMDN_ERR_INVALID, "null pointer");
  if (reinterpret_cast<uintptr_t>(dy) % 16)
    return fail(GMDN_ERR_INVALID, "head_rmsnorm: pointers must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float e = eps < 0.f ? 1.1920928955078125e-07f : eps;
  if (static_cast<long long>(B) * H * T == 0) {
    cudaError_t ce = cudaMemsetAsync(dweight, 0, sizeof(float) * dh, st);
    return ce == cudaSuccess ? GMDN_OK : cuda_fail(ce, "head_rmsnorm_bwd");
  }
  GMDN_LAUNCH(gmdn::head_rmsnorm_bwd(o, weight, dy, d_o, dweight, B, H, T, dh, e, in_f32 != 0,
                                     out_f32 != 0, st),
              "head_rmsnorm_bwd");
  return GMDN_OK;
}

void gmdn_prof_enable(int on) { g_prof_on.store(on ? 1 : 0); }

const char* gmdn_prof_report(void) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  std::map<std::string, std::pair<double, int>> agg;
  for (auto& r : g_prof_recs) {
    float ms = 0.f;
    if (cudaEventSynchronize(r.stop) == cudaSuccess &&
        cudaEventElapsedTime(&ms, r.start, r.stop) == cudaSuccess) {
      auto& e = agg[r.name];
      e.first += ms;
      e.second += 1;
    }
    g_prof_pool.push_back(r.start);
    g_prof_pool.push_back(r.stop);
  }
  g_prof_recs.clear();
  std::string js = "{";
  bool first = true;
  for (auto& kv : agg) {
    char buf[256];
    snprintf(buf, sizeof(buf), "%s\"%s\": [%.6f, %d]", first ? "" : ", ", kv.first.c_str(),
             kv.second.first, kv.second.second);
    js += buf;
    first = false;
  }
  js += "}";
  g_prof_json = js;
  return g_prof_json.c_str();
}

size_t gmdn_scan_saved_bytes(int B, int H, int N, int dh, int rule) {
  if (B < 0 || H < 0 || N < 0 || !dh_ok(dh)) return 0;
  return carve_scan_saved(nullptr, B * H, N, dh, rule).bytes;
}

// The scan workspace: the device status word (first 256 bytes, read by
// gmdn_chunk_status), then the exact-fp32 kernels' per-(b,h) scratch.
constexpr size_t kScanStatusBytes = 256;

size_t gmdn_scan_workspace_bytes(int B, int H, int N, int dh, int rule, int ns, int precision) {
  (void)N;
  (void)rule;
  (void)precision;
  if (B < 0 || H < 0 || !dh_ok(dh) || ns < 0) return 0;
  return kScanStatusBytes + align_up(scan_scratch_floats(B * H, dh, ns) * sizeof(float));
}

int gmdn_scan_fwd(const float* U, const float* K, const float* a, const float* b,
                  const float* m, const float* n, float* S_out, void* saved,
                  void* workspace, size_t workspace_bytes, int B, int H, int N, int dh,
                  int rule, int ns, int precision, void* stream) {
  g_last_error.clear();
  int rc = check_common(B, H, N, dh, rule, ns, precision);
  if (rc) return rc;
  if (B * H * N == 0) return GMDN_OK;
  if (!U || !K || !a || !b || !m || !n || !S_out)
    return fail(GMDN_ERR_INVALID, "null input/output pointer");
  if (rule != 0 && !saved) return fail(GMDN_ERR_INVALID, "muon/adam need the saved buffer");
  const size_t need = gmdn_scan_workspace_bytes(B, H, N, dh, rule, ns, precision);
  if (!workspace || workspace_bytes < need)
    return fail(GMDN_ERR_WORKSPACE, "workspace %zu bytes < required %zu", workspace_bytes, need);
  ScanSaved sv = carve_scan_saved(saved, B * H, N, dh, rule);
  gmdn::ScanArgs p{};
  p.U = U; p.K = K; p.a = a; p.b = b; p.m = m; p.n = n;
  p.S = S_out; p.M_hist = sv.M_hist; p.V_hist = sv.V_hist;
  p.scratch = reinterpret_cast<float*>(static_cast<char*>(workspace) + kScanStatusBytes);
  p.BH = B * H; p.N = N; p.dh = dh; p.rule = rule; p.ns = ns;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t* status = static_cast<uint32_t*>(workspace);
  cudaError_t e = cudaMemsetAsync(status, 0, sizeof(uint32_t), st);
  if (e != cudaSuccess) return cuda_fail(e, "status reset");
  // GMDN_PREC_FAST, delta at dh 128 with 16-byte aligned tensors: the
  // tensor-core scan (its bounded waits report through the status word);
  // everything else runs the exact-fp32 kernels.
  if (precision == GMDN_PREC_FAST && gmdn::scan_fwd_tc_supported(p)) {
    GMDN_LAUNCH(gmdn::scan_fwd_tc(p, status, st), "scan_fwd_tc");
    return GMDN_OK;
  }
  GMDN_LAUNCH(gmdn::scan_fwd_ieee(p, st), "scan_fwd_ieee");
  return GMDN_OK;
}

int gmdn_scan_bwd(const float* U, const float* K, const float* a, const float* b,
                  const float* m, const float* n, const float* S_all, const void* saved,
                  const float* gS, float* dU, float* dK, float* da, float* db, float* dm,
                  float* dn, void* workspace, size_t workspace_bytes, int B, int H, int N,
                  int dh, int rule, int ns, int precision, void* stream) {
  g_last_error.clear();
  int rc = check_common(B, H, N, dh, rule, ns, precision);
  if (rc) return rc;
  if (B * H * N == 0) return GMDN_OK;
  if (!U || !K || !a || !b || !m || !n || !S_all || !gS || !dU || !dK || !da || !db || !dm ||
      !dn)
    return fail(GMDN_ERR_INVALID, "null input/output pointer");
  if (rule != 0 && !saved) return fail(GMDN_ERR_INVALID, "muon/adam need the saved buffer");
  const size_t need = gmdn_scan_workspace_bytes(B, H, N, dh, rule, ns, precision);
  if (!workspace || workspace_bytes < need)
    return fail(GMDN_ERR_WORKSPACE, "workspace %zu bytes < required %zu", workspace_bytes, need);
  ScanSaved sv = carve_scan_saved(const_cast<void*>(saved), B * H, N, dh, rule);
  gmdn::ScanArgs p{};
  p.U = U; p.K = K; p.a = a; p.b = b; p.m = m; p.n = n;
  p.S = const_cast<float*>(S_all); p.M_hist = sv.M_hist; p.V_hist = sv.V_hist;
  p.gS = gS; p.dU = dU; p.dK = dK; p.da = da; p.db = db; p.dm = dm; p.dn = dn;
  p.scratch = reinterpret_cast<float*>(static_cast<char*>(workspace) + kScanStatusBytes);
  p.BH = B * H; p.N = N; p.dh = dh; p.rule = rule; p.ns = ns;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t* status = static_cast<uint32_t*>(workspace);
  cudaError_t e = cudaMemsetAsync(status, 0, sizeof(uint32_t), st);
  if (e != cudaSuccess) return cuda_fail(e, "status reset");
  // GMDN_PREC_FAST, delta at dh 128: the reverse chain on the tensor cores,
  // then dK and da for every matrix
  if (precision == GMDN_PREC_FAST && gmdn::scan_bwd_tc_supported(p)) {
    GMDN_LAUNCH(gmdn::scan_bwd_chain_tc(p, status, st), "scan_bwd_chain_tc");
    GMDN_LAUNCH(gmdn::scan_bwd_dk_tc(p, status, st), "scan_bwd_dk_tc");
    return GMDN_OK;
  }
  GMDN_LAUNCH(gmdn::scan_bwd_ieee(p, st), "scan_bwd_ieee");
  return GMDN_OK;
}

size_t gmdn_chunk_saved_bytes_ex(int B, int H, int T, int dh, int chunk, int rule, int ns,
                                 int precision, int io_f32) {
  if (B < 0 || H < 0 || T < 0 || !dh_ok(dh) || chunk <= 0) return 0;
  const int N = T / chunk;
  return carve_chunk(nullptr, nullptr, B * H, N, dh, rule, ns,
                     chunk_fast(dh, chunk, rule, precision, io_f32, N)).saved_bytes;
}

size_t gmdn_chunk_workspace_bytes_ex(int B, int H, int T, int dh, int chunk, int rule, int ns,
                                     int precision, int io_f32) {
  if (B < 0 || H < 0 || T < 0 || !dh_ok(dh) || chunk <= 0 || ns < 0) return 0;
  const int N = T / chunk;
  return carve_chunk(nullptr, nullptr, B * H, N, dh, rule, ns,
                     chunk_fast(dh, chunk, rule, precision, io_f32, N)).ws_bytes;
}

size_t gmdn_chunk_saved_bytes(int B, int H, int T, int dh, int chunk, int rule, int ns,
                              int precision) {
  return gmdn_chunk_saved_bytes_ex(B, H, T, dh, chunk, rule, ns, precision, 0);
}

size_t gmdn_chunk_workspace_bytes(int B, int H, int T, int dh, int chunk, int rule, int ns,
                                  int precision) {
  return gmdn_chunk_workspace_bytes_ex(B, H, T, dh, chunk, rule, ns, precision, 0);
}

int gmdn_chunk_status(const void* workspace, void* stream) {
  g_last_error.clear();
  if (!workspace) return fail(GMDN_ERR_INVALID, "null workspace");
  uint32_t v = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(&v, workspace, sizeof(v), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "gmdn_chunk_status");
  if (v) return fail(GMDN_ERR_DEVICE, "kernel status word 0x%x (1 = a wait timed out)", v);
  return GMDN_OK;
}

static int chunk_setup(gmdn::ChunkArgs& p, ChunkBufs& bufs, const void* q, const void* k,
                       const void* v, const float* alpha, const float* beta, const float* mu,
                       const float* nu, void* saved, void* workspace, size_t workspace_bytes,
                       int B, int H, int T, int dh, int chunk, int rule, int ns, int precision,
                       int io_f32, bool* fast) {
  int rc = check_chunk(B, H, T, dh, chunk, rule, ns, precision);
  if (rc) return rc;
  if (!q || !k || !v || !alpha || !beta || !mu) return fail(GMDN_ERR_INVALID, "null input pointer");
  if (rule == 2 && !nu) return fail(GMDN_ERR_INVALID, "adam (rule 2) needs nu");
  if (!saved) return fail(GMDN_ERR_INVALID, "null saved buffer");
  const int N = T / chunk;
  *fast = chunk_fast(dh, chunk, rule, precision, io_f32, N);
  bufs = carve_chunk(saved, workspace, B * H, N, dh, rule, ns, *fast);
  if (!workspace || workspace_bytes < bufs.ws_bytes)
    return fail(GMDN_ERR_WORKSPACE, "workspace %zu bytes < required %zu", workspace_bytes,
                bufs.ws_bytes);
  p = gmdn::ChunkArgs{};
  p.q = q; p.k = k; p.v = v;
  p.alpha = alpha; p.beta = beta; p.mu = mu; p.nu = (rule == 2) ? nu : nullptr;
  p.Kw = bufs.Kw; p.Uv = bufs.Uv; p.S = bufs.S; p.gS = bufs.gS; p.dUv = bufs.dUv;
  p.dKw = bufs.dKw;
  p.a_c = bufs.a_c; p.b_c = bufs.b_c; p.m_c = bufs.m_c; p.n_c = bufs.n_c;
  p.da_c = bufs.da_c; p.db_c = bufs.db_c; p.dm_c = bufs.dm_c; p.dn_c = bufs.dn_c;
  p.BH = B * H; p.T = T; p.N = N; p.C = chunk; p.dh = dh; p.rule = rule;
  p.io_f32 = io_f32 != 0;
  return GMDN_OK;
}

static gmdn::ScanArgs scan_args_from(const gmdn::ChunkArgs& c, const ChunkBufs& b, int ns) {
  gmdn::ScanArgs s{};
  s.U = b.Uv; s.K = b.Kw; s.a = b.a_c; s.b = b.b_c; s.m = b.m_c; s.n = b.n_c;
  s.S = b.S; s.M_hist = b.M_hist; s.V_hist = b.V_hist;
  s.gS = b.gS; s.dU = b.dUv; s.dK = b.dKw;
  s.da = b.da_c; s.db = b.db_c; s.dm = b.dm_c; s.dn = b.dn_c;
  s.scratch = b.scratch;
  s.BH = c.BH; s.N = c.N; s.dh = c.dh; s.rule = c.rule; s.ns = ns;
  return s;
}

int gmdn_chunk_fwd_ex(const void* q, const void* k, const void* v, const float* alpha,
                      const float* beta, const float* mu, const float* nu, void* o, void* saved,
                      void* workspace, size_t workspace_bytes, int B, int H, int T, int dh,
                      int chunk, int rule, int ns, int precision, int io_f32, void* stream) {
  g_last_error.clear();
  if (B * H * T == 0) return check_chunk(B, H, T, dh, chunk, rule, ns, precision);
  gmdn::ChunkArgs p;
  ChunkBufs bufs;
  bool fast = false;
  int rc = chunk_setup(p, bufs, q, k, v, alpha, beta, mu, nu, saved, workspace, workspace_bytes,
                       B, H, T, dh, chunk, rule, ns, precision, io_f32, &fast);
  if (rc) return rc;
  if (!o) return fail(GMDN_ERR_INVALID, "null output pointer");
  p.o = o;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(bufs.status, 0, sizeof(uint32_t), st);
  if (e != cudaSuccess) return cuda_fail(e, "status reset");
  if (fast) {
    if (rule == 1)
      GMDN_LAUNCH(gmdn::chunk_fwd_muon_tc(p, bufs.tc, ns, st), "chunk_fwd_muon_tc");
    else
      GMDN_LAUNCH(gmdn::chunk_fwd_tc(p, bufs.tc, st), "chunk_fwd_tc");
    return GMDN_OK;
  }
  gmdn::ScanArgs sp = scan_args_from(p, bufs, ns);
  GMDN_LAUNCH(gmdn::chunk_prep_ieee(p, st), "chunk_prep");
  GMDN_LAUNCH(gmdn::scan_fwd_ieee(sp, st), "scan_fwd_ieee");
  GMDN_LAUNCH(gmdn::chunk_out_ieee(p, st), "chunk_out");
  return GMDN_OK;
}

int gmdn_chunk_bwd_ex(const void* q, const void* k, const void* v, const float* alpha,
                      const float* beta, const float* mu, const float* nu, const void* dO,
                      const void* saved, void* dq, void* dk, void* dv, float* dalpha,
                      float* dbeta, float* dmu, float* dnu, void* workspace,
                      size_t workspace_bytes, int B, int H, int T, int dh, int chunk, int rule,
                      int ns, int precision, int io_f32, void* stream) {
  g_last_error.clear();
  if (B * H * T == 0) return check_chunk(B, H, T, dh, chunk, rule, ns, precision);
  gmdn::ChunkArgs p;
  ChunkBufs bufs;
  bool fast = false;
  int rc = chunk_setup(p, bufs, q, k, v, alpha, beta, mu, nu, const_cast<void*>(saved),
                       workspace, workspace_bytes, B, H, T, dh, chunk, rule, ns, precision,
                       io_f32, &fast);
  if (rc) return rc;
  if (!dO || !dq || !dk || !dv || !dalpha || !dbeta || !dmu)
    return fail(GMDN_ERR_INVALID, "null gradient pointer");
  if (rule == 2 && !dnu) return fail(GMDN_ERR_INVALID, "adam (rule 2) needs dnu");
  p.dO = dO; p.dq = dq; p.dk = dk; p.dv = dv;
  p.dalpha = dalpha; p.dbeta = dbeta; p.dmu = dmu; p.dnu = dnu;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(bufs.status, 0, sizeof(uint32_t), st);
  if (e != cudaSuccess) return cuda_fail(e, "status reset");
  if (fast) {
    const int n_fused = rule == 0 ? gmdn::chunk_bwd_fused_tiles(p) : 0;
    if (n_fused > 0) {
      GMDN_LAUNCH(gmdn::chunk_bwd_fused_tc(p, bufs.tc, n_fused, st), "chunk_bwd_fused_tc");
      if (n_fused < p.BH * p.N)
        GMDN_LAUNCH(gmdn::chunk_bwd2_tc(p, bufs.tc, st, n_fused), "chunk_bwd2_tc");
      return GMDN_OK;
    }
    if (rule == 1)
      GMDN_LAUNCH(gmdn::chunk_bwd1_muon_tc(p, bufs.tc, ns, st), "chunk_bwd1_muon_tc");
    else
      GMDN_LAUNCH(gmdn::chunk_bwd1_tc(p, bufs.tc, st), "chunk_bwd1_tc");
    GMDN_LAUNCH(gmdn::chunk_bwd2_tc(p, bufs.tc, st), "chunk_bwd2_tc");
    return GMDN_OK;
  }
  gmdn::ScanArgs sp = scan_args_from(p, bufs, ns);
  // Kw, Uv and the chunk gate products are recomputed rather than saved.
  GMDN_LAUNCH(gmdn::chunk_prep_ieee(p, st), "chunk_prep");
  GMDN_LAUNCH(gmdn::chunk_state_grad_ieee(p, st), "chunk_state_grad");
  GMDN_LAUNCH(gmdn::scan_bwd_ieee(sp, st), "scan_bwd_ieee");
  GMDN_LAUNCH(gmdn::chunk_token_grad_ieee(p, st), "chunk_token_grad");
  return GMDN_OK;
}

int gmdn_chunk_fwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* alpha,
                   const float* beta, const float* mu, const float* nu, uint16_t* o, void* saved,
                   void* workspace, size_t workspace_bytes, int B, int H, int T, int dh,
                   int chunk, int rule, int ns, int precision, void* stream) {
  return gmdn_chunk_fwd_ex(q, k, v, alpha, beta, mu, nu, o, saved, workspace, workspace_bytes,
                           B, H, T, dh, chunk, rule, ns, precision, 0, stream);
}

int gmdn_chunk_bwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* alpha,
                   const float* beta, const float* mu, const float* nu, const uint16_t* dO,
                   const void* saved, uint16_t* dq, uint16_t* dk, uint16_t* dv, float* dalpha,
                   float* dbeta, float* dmu, float* dnu, void* workspace,
                   size_t workspace_bytes, int B, int H, int T, int dh, int chunk, int rule,
                   int ns, int precision, void* stream) {
  return gmdn_chunk_bwd_ex(q, k, v, alpha, beta, mu, nu, dO, saved, dq, dk, dv, dalpha, dbeta,
                           dmu, dnu, workspace, workspace_bytes, B, H, T, dh, chunk, rule, ns,
                           precision, 0, stream);
}

}  // extern "C"

// ---- allocation-free variant of gmdn_scan_fwd --------------------------------
//
// Scratch of the exact-fp32 scan forward for callers that cannot allocate
// device memory (their runtime hands a call only its operand and result
// buffers).  One file-scope array per device: every GPU that loads this
// library holds GMDN_NOALLOC_SCRATCH_BYTES of it until the process exits.  In
// host code `g_noalloc_scratch` names the symbol only; its device address
// comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[GMDN_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kNoallocMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device.  The first call
// on a device looks it up (which may load this library's device code onto that
// device); later calls read the cached pointer.
int noalloc_scratch(float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kNoallocMaxDevices)
    return fail(GMDN_ERR_DEVICE, "device ordinal %d beyond the %d the static scratch tracks",
                dev, kNoallocMaxDevices);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static scan scratch)");
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return GMDN_OK;
}

}  // namespace

extern "C" {

int gmdn_scan_fwd_noalloc(const float* U, const float* K, const float* a, const float* b,
                          const float* m, const float* n, float* S_out, void* saved, int B,
                          int H, int N, int dh, int rule, int ns, int precision,
                          void* stream) {
  g_last_error.clear();
  int rc = check_common(B, H, N, dh, rule, ns, precision);
  if (rc) return rc;
  if (B * H * N == 0) return GMDN_OK;
  if (!U || !K || !a || !b || !m || !n || !S_out)
    return fail(GMDN_ERR_INVALID, "null input/output pointer");
  if (rule != 0 && !saved) return fail(GMDN_ERR_INVALID, "muon/adam need the saved buffer");
  // The forward kernel uses kScanFwdScratchMats dh x dh fp32 matrices per (b,h).
  const size_t per_bh = mats(gmdn::kScanFwdScratchMats, dh) * sizeof(float);
  const size_t need = static_cast<size_t>(B) * H * per_bh;
  if (need > GMDN_NOALLOC_SCRATCH_BYTES)
    return fail(GMDN_ERR_WORKSPACE,
                "gmdn_scan_fwd_noalloc: B*H = %d at dh = %d needs %zu scratch bytes, more than "
                "the %zu-byte static scratch (at most %zu (b,h) pairs at this dh); call "
                "gmdn_scan_fwd with a workspace instead",
                B * H, dh, need, static_cast<size_t>(GMDN_NOALLOC_SCRATCH_BYTES),
                static_cast<size_t>(GMDN_NOALLOC_SCRATCH_BYTES) / per_bh);
  float* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  ScanSaved sv = carve_scan_saved(saved, B * H, N, dh, rule);
  gmdn::ScanArgs p{};
  p.U = U; p.K = K; p.a = a; p.b = b; p.m = m; p.n = n;
  p.S = S_out; p.M_hist = sv.M_hist; p.V_hist = sv.V_hist;
  p.scratch = scratch;
  p.BH = B * H; p.N = N; p.dh = dh; p.rule = rule; p.ns = ns;
  // The kernel zeroes its state and moment matrices before the first chunk and
  // writes every other scratch matrix before reading it, so what an earlier
  // call left in the array never reaches the result.
  cudaError_t e = gmdn::scan_fwd_ieee(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "scan_fwd_ieee (static scratch)");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return GMDN_OK;
}

}  // extern "C"
