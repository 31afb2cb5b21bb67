// api.cu -- the extern "C" entry points declared in include/semicrf.h.
//
// Every entry point validates its arguments, carves the caller-provided
// workspace, and enqueues kernels on the given stream.  No device memory is
// allocated here and nothing synchronises.

#include <cmath>
#include <cstring>

#include <algorithm>

#include "semicrf_internal.cuh"

using namespace semicrf;

int semicrf::device_sm_count() {
  constexpr int kMaxDev = 64;
  static int cache[kMaxDev] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
  if (dev < kMaxDev && cache[dev] > 0) return cache[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;  // no device answer: the B200's count, for planning only
  if (dev < kMaxDev) cache[dev] = n;
  return n;
}

namespace {

constexpr int kP = 8;  // chain block size (chain_block_size)

struct Carver {
  char* base;
  size_t off = 0;
  explicit Carver(void* p) : base(static_cast<char*>(p)) {}
  template <class T>
  T* take(size_t n) {
    off = (off + 255) & ~size_t(255);
    T* r = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += n * sizeof(T);
    return r;
  }
  size_t bytes() const { return (off + 255) & ~size_t(255); }
};

int kcap_of(int64_t K) { return K > 1 ? (int)(K - 1) : 1; }
int sint_of(const semicrf_problem* p) {
  const int64_t S = p->checkpoint_interval;
  return (int)(((S + kP - 1) / kP) * kP);
}
int nint_of(const semicrf_problem* p) { return (int)(p->T / sint_of(p) + 1); }

// shape-level checks (used by the size queries, which take no pointers)
int validate_shape(const semicrf_problem* p) {
  if (!p) return SEMICRF_ERR_INVALID_ARGUMENT;
  if (p->batch < 0 || p->T < 0 || p->K < 1 || p->C < 1) return SEMICRF_ERR_INVALID_ARGUMENT;
  if (p->semiring != SEMICRF_LOG && p->semiring != SEMICRF_MAX) return SEMICRF_ERR_SEMIRING;
  if (p->transition_ndim != 2 && p->transition_ndim != 3) return SEMICRF_ERR_INVALID_ARGUMENT;
  if (p->checkpoint_interval < p->K) return SEMICRF_ERR_INVALID_ARGUMENT;
  if (p->C > 256 || p->T > (int64_t)1 << 30 || p->K > 32767) return SEMICRF_ERR_UNSUPPORTED;
  if (p->backward_mode != SEMICRF_KEEP_ALPHA && p->backward_mode != SEMICRF_RECOMPUTE)
    return SEMICRF_ERR_INVALID_ARGUMENT;
  if (p->transition_ndim == 3)  // duration-dependent transitions: kcc.cu
    return kcc_supported((int)p->C, (int)p->K) ? SEMICRF_OK : SEMICRF_ERR_UNSUPPORTED;
  if (p->semiring == SEMICRF_LOG && !lchain_supported((int)p->C, (int)p->K))
    return SEMICRF_ERR_UNSUPPORTED;
  if (p->semiring == SEMICRF_LOG && !lmarg_plan(1, 1, (int)p->K, (int)p->C).ok)
    return SEMICRF_ERR_UNSUPPORTED;
  if (!chain_supported((int)p->C, (int)p->K, SEMICRF_MAX, true)) return SEMICRF_ERR_UNSUPPORTED;
  return SEMICRF_OK;
}

int validate(const semicrf_problem* p) {
  const int st = validate_shape(p);
  if (st != SEMICRF_OK) return st;
  if (p->batch > 0 && (!p->cum_scores || !p->transition || !p->duration_bias || !p->lengths))
    return SEMICRF_ERR_INVALID_ARGUMENT;
  return SEMICRF_OK;
}

Prepared carve_prep(Carver& cv, int C, int K, int semiring) {
  Prepared pr{};
  const int kx = kcap_of(K) + kPrepRowsExtra;
  if (semiring == SEMICRF_LOG) {
    pr.mxd_f = cv.take<double>((size_t)C * C);
    pr.mxd_b = cv.take<double>((size_t)C * C);
    pr.dbed = cv.take<double>((size_t)kx * C);
    pr.ovf = cv.take<int>(1);
  } else {
    pr.mx_f = cv.take<float>((size_t)C * C);
    pr.mx_b = cv.take<float>((size_t)C * C);
  }
  pr.colmax_f = cv.take<float>(C);
  pr.colmax_b = cv.take<float>(C);
  pr.dbl = cv.take<float>((size_t)kx * C);
  pr.dbmax = cv.take<float>(C);
  pr.kx = kx;
  return pr;
}

struct SavedLayout {
  double* logz;
  float* sv_f;     // max semiring: float32 restart records
  double* sv_d;
  double* sv;      // log semiring, SEMICRF_RECOMPUTE: float64 restart records
  double* a_tab;   // log semiring, SEMICRF_KEEP_ALPHA: alpha tables
  double* A_tab;
  double* n_tab;
  double* b_tab;   // ... and the beta chain's tables
  double* B_tab;
  double* m_tab;
  ChunkPlan cp;    // time chunks of the two chains (keep mode)
  double *hand_a, *hand_b, *rdiff, *dofs;
  int *okf, *fail;
  int* redo;       // [2][B]: the sequences whose chunks rerun with the second warm-up
  int* rec_ovf;    // SEMICRF_RECOMPUTE: set when the forward's float64 frames clipped
};

ChunkPlan keep_chunk_plan(const semicrf_problem* p) {
  if (p->semiring != SEMICRF_LOG || p->backward_mode != SEMICRF_KEEP_ALPHA ||
      !lchain_ws_supported((int)p->C, (int)p->K))
    return ChunkPlan{1, (int)p->T, 0, 0};
  return chunk_plan((int)p->batch, (int)p->T, (int)p->K, (int)p->C, 2, p->chunk_warmup);
}

SavedLayout carve_saved(Carver& cv, const semicrf_problem* p) {
  SavedLayout s{};
  const size_t B = p->batch, C = p->C;
  const size_t kc = kcap_of(p->K), nint = nint_of(p);
  s.logz = cv.take<double>(B);
  if (p->transition_ndim == 3) {
    // (K, C, C): log alpha, its row maxima and log beta, whatever the mode
    const size_t n = B * (p->T + 1) * C;
    s.a_tab = cv.take<double>(n);
    s.n_tab = cv.take<double>(B * (p->T + 1));
    s.b_tab = cv.take<double>(n);
  } else if (p->semiring == SEMICRF_MAX) {
    s.sv_f = cv.take<float>(B * nint * (kc * C + 2 * C));
    s.sv_d = cv.take<double>(B * nint * kc);
  } else if (p->backward_mode == SEMICRF_RECOMPUTE) {
    s.sv = cv.take<double>(B * nint * lchain_saved_doubles((int)p->C, (int)p->K));
    s.rec_ovf = cv.take<int>(1);
  } else {
    const size_t n = B * (p->T + 1) * C;
    s.a_tab = cv.take<double>(n);
    s.A_tab = cv.take<double>(n);
    s.n_tab = cv.take<double>(B * (p->T + 1));
    s.b_tab = cv.take<double>(n);
    s.B_tab = cv.take<double>(n);
    s.m_tab = cv.take<double>(B * (p->T + 1));
    s.cp = keep_chunk_plan(p);
    if (s.cp.nchunk > 1) {
      const size_t nh = chunk_hand_doubles((int)B, (int)p->K, (int)C, s.cp);
      const size_t nc = B * s.cp.nchunk;
      s.hand_a = cv.take<double>(nh);
      s.hand_b = cv.take<double>(nh);
      s.rdiff = cv.take<double>(2 * nc);
      s.dofs = cv.take<double>(2 * nc);
      s.okf = cv.take<int>(2 * nc);
      s.fail = cv.take<int>(2 * B);
      s.redo = cv.take<int>(2 * B);
    }
  }
  return s;
}

ChainArgs base_args(const semicrf_problem* p) {
  ChainArgs a{};
  a.cum = p->cum_scores;
  a.ps = p->proj_start;
  a.pe = p->proj_end;
  a.lengths = p->lengths;
  return a;
}

ChainLaunch base_launch(const semicrf_problem* p, const Prepared& pr) {
  ChainLaunch L{};
  L.B = (int)p->batch;
  L.T = (int)p->T;
  L.K = (int)p->K;
  L.C = (int)p->C;
  L.kcap = kcap_of(p->K);
  L.prep = pr;
  return L;
}

struct BwdLayout {
  Prepared pr;
  float *xa, *ma, *xb, *mb, *pstart, *alse, *part_tr, *part_db;
  double *na, *nb;
};

struct LBwdLayout {
  Prepared pr;
  double *a_tab, *A_tab, *n_tab;  // SEMICRF_RECOMPUTE: alpha tables
  double *b_tab, *B_tab, *m_tab;  // SEMICRF_RECOMPUTE: beta tables
  double *la, *lb, *maX, *mbY, *part_tr, *part_db;
  int* dbflag;
  LMargPlan mp;
};

LBwdLayout carve_lbwd(Carver& cv, const semicrf_problem* p) {
  LBwdLayout w{};
  w.pr = carve_prep(cv, (int)p->C, (int)p->K, p->semiring);
  const size_t n = (size_t)p->batch * (p->T + 1) * p->C;
  const size_t nt = (size_t)p->batch * (p->T + 1);
  if (p->backward_mode == SEMICRF_RECOMPUTE) {
    w.a_tab = cv.take<double>(n);
    w.A_tab = cv.take<double>(n);
    w.n_tab = cv.take<double>(nt);
    w.b_tab = cv.take<double>(n);
    w.B_tab = cv.take<double>(n);
    w.m_tab = cv.take<double>(nt);
  }
  w.mp = lmarg_plan((int)p->batch, (int)p->T, (int)p->K, (int)p->C);
  w.la = cv.take<double>(n);
  w.lb = cv.take<double>(n);
  w.maX = cv.take<double>((size_t)p->batch * w.mp.nblk * p->C);
  w.mbY = cv.take<double>((size_t)p->batch * w.mp.nblk * p->C);
  w.part_tr = cv.take<double>((size_t)p->batch * w.mp.nchunk * p->C * p->C);
  w.part_db = cv.take<double>((size_t)p->batch * w.mp.nsplit * kcap_of(p->K) * p->C);
  w.dbflag = cv.take<int>((size_t)p->batch);
  return w;
}

// Both chains of every sequence in time chunks (one CTA per chunk and chain),
// then the boundary check and offset fix-up per chain; when the plan has a
// second warm-up, the chunks of sequences that did not join again with it and
// their boundaries checked again; then a serial rerun of any sequence whose
// chunks still did not join.
cudaError_t chunked_chains(const semicrf_problem* p, LChainLaunch L, const SavedLayout& sl,
                           cudaStream_t s) {
  const int B = (int)p->batch, P = sl.cp.nchunk;
  for (LChainArgs* a : {&L.a0, &L.a1}) {
    a->nchunk = P;
    a->chunk_len = sl.cp.len;
    a->warm = sl.cp.warm;
  }
  L.a0.hand = sl.hand_a;
  L.a1.hand = sl.hand_b;
  L.n1 = B * P;
  cudaError_t e = launch_lchain_ws(L, 2 * B * P, s);
  if (e != cudaSuccess) return e;
  auto fix_all = [&](const int* only) -> cudaError_t {
    ChunkFix fr[2];
    for (int role = 0; role < 2; ++role) {
      ChunkFix& f = fr[role];
      f = ChunkFix{};
      f.B = B;
      f.T = (int)p->T;
      f.K = (int)p->K;
      f.C = (int)p->C;
      f.dir = role;
      f.cp = sl.cp;
      f.lengths = p->lengths;
      f.hand = role ? sl.hand_b : sl.hand_a;
      f.rdiff = sl.rdiff + (size_t)role * B * P;
      f.okf = sl.okf + (size_t)role * B * P;
      f.D = sl.dofs + (size_t)role * B * P;
      f.fail = sl.fail + (size_t)role * B;
      f.only = only ? only + (size_t)role * B : nullptr;
      f.n_tab = role ? sl.m_tab : sl.n_tab;
      f.logz = role ? nullptr : L.a0.logz;
      f.partition = role ? nullptr : L.a0.partition;
    }
    return launch_chunk_fix(fr[0], fr[1], s);
  };
  e = fix_all(nullptr);
  if (e != cudaSuccess) return e;
  if (sl.cp.warm2 > 0) {
    // sequences whose boundaries did not join: their chunks again with the
    // longer warm-up, then their boundaries checked again (the others are
    // final and untouched: the chains skip them, the fix-up ignores them)
    if (cudaMemcpyAsync(sl.redo, sl.fail, 2 * (size_t)B * sizeof(int),
                        cudaMemcpyDeviceToDevice, s) != cudaSuccess)
      return cudaErrorUnknown;
    LChainLaunch L2 = L;
    L2.a0.warm = L2.a1.warm = sl.cp.warm2;
    L2.a0.only = sl.redo;
    L2.a1.only = sl.redo + B;
    e = launch_lchain_ws(L2, 2 * B * P, s);
    if (e != cudaSuccess) return e;
    e = fix_all(sl.redo);
    if (e != cudaSuccess) return e;
  }
  // sequences whose chunks did not join: each chain again, whole
  for (LChainArgs* a : {&L.a0, &L.a1}) {
    a->nchunk = 1;
    a->hand = nullptr;
  }
  L.a0.only = sl.fail;
  L.a1.only = sl.fail + B;
  L.n1 = B;
  return launch_lchain_ws(L, 2 * B, s);
}

// the beta chain (dir 1) of a log-semiring problem, writing its tables
LChainArgs beta_chain_args(const semicrf_problem* p, const Prepared& pr, double* b_tab,
                           double* B_tab, double* m_tab) {
  LChainArgs a{};
  a.mode = 0;
  a.dir = 1;
  a.cum = p->cum_scores;
  a.ps = p->proj_start;
  a.pe = p->proj_end;
  a.lengths = p->lengths;
  a.mx = pr.mxd_b;
  a.colmax = pr.colmax_b;
  a.a_tab = b_tab;
  a.A_tab = B_tab;
  a.n_tab = m_tab;
  return a;
}

BwdLayout carve_bwd(Carver& cv, const semicrf_problem* p) {
  BwdLayout w{};
  w.pr = carve_prep(cv, (int)p->C, (int)p->K, p->semiring);
  const size_t n = (size_t)p->batch * (p->T + 1) * p->C;
  const size_t nt = (size_t)p->batch * (p->T + 1);
  w.xa = cv.take<float>(n);
  w.ma = cv.take<float>(n);
  w.xb = cv.take<float>(n);
  w.mb = cv.take<float>(n);
  w.pstart = cv.take<float>(n);
  w.alse = p->semiring == SEMICRF_MAX ? cv.take<float>(n) : nullptr;
  w.na = cv.take<double>(nt);
  w.nb = cv.take<double>(nt);
  w.part_tr = cv.take<float>((size_t)p->batch * p->C * p->C);
  w.part_db = cv.take<float>((size_t)p->batch * p->K * p->C);
  return w;
}

struct VitLayout {
  Prepared pr;
  int16_t* bp_k;
  uint8_t* bp_c;
  uint16_t* bp;  // packed backpointers of the warp chain
  int* final_c;
};

VitLayout carve_vit(Carver& cv, const semicrf_problem* p) {
  VitLayout w{};
  w.pr = carve_prep(cv, (int)p->C, (int)p->K, p->semiring);
  const size_t n = (size_t)p->batch * (p->T + 1) * p->C;
  w.bp_k = cv.take<int16_t>(n);
  w.bp_c = cv.take<uint8_t>(n);
  w.bp = cv.take<uint16_t>(n);
  w.final_c = cv.take<int>(p->batch);
  return w;
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? SEMICRF_OK : SEMICRF_ERR_CUDA; }

// (K, C, C) transitions: prepared factors, then (backward) the marginal terms
struct KccLayout {
  KccPrep pr;
  double *st, *et, *pend, *part_tr, *al, *anc, *ep1;
  int* kflag;
  int nslice;
};

KccLayout carve_kcc(Carver& cv, const semicrf_problem* p, bool backward) {
  KccLayout w{};
  const int K = (int)p->K, C = (int)p->C;
  w.pr = kcc_prep_carve(cv.take<double>(kcc_prep_doubles(K, C, p->semiring)), K, C,
                        p->semiring);
  // the blocked kernels' overflow flag (forward: chain; backward: gradients)
  if (kblk_supported(C, K)) w.kflag = cv.take<int>(1);
  if (!backward) return w;
  const size_t n = (size_t)p->batch * (p->T + 1) * p->C;
  w.st = cv.take<double>(n);
  w.et = cv.take<double>(n);
  w.pend = p->semiring == SEMICRF_MAX ? cv.take<double>(n) : nullptr;
  const bool blk = kblk_supported(C, K);  // blocked gradient kernels (both semirings)
  if (blk) {
    w.al = cv.take<double>(n);
    w.ep1 = cv.take<double>(n);
    w.anc = cv.take<double>((size_t)p->batch * kblk_anchor_rows((int)p->T) * C);
  }
  w.nslice = blk ? kblk_tr_slices((int)p->batch, K, C) : kcc_tr_slices((int)p->batch, K, C);
  // room for the per-item kernels' slices too: they are the blocked path's fallback
  const int nsl_all = std::max(w.nslice, kcc_tr_slices((int)p->batch, K, C));
  w.part_tr = cv.take<double>((size_t)nsl_all * C * (size_t)(K - 1) * C);
  return w;
}

KccArgs kcc_args(const semicrf_problem* p, const KccPrep& pr) {
  KccArgs a{};
  a.B = (int)p->batch;
  a.T = (int)p->T;
  a.K = (int)p->K;
  a.C = (int)p->C;
  a.kcap = kcap_of(p->K);
  a.semiring = p->semiring;
  a.cum = p->cum_scores;
  a.tr = p->transition;
  a.db = p->duration_bias;
  a.ps = p->proj_start;
  a.pe = p->proj_end;
  a.lengths = p->lengths;
  a.pr = pr;
  return a;
}

VChainArgs vchain_args(const semicrf_problem* p) {
  VChainArgs v{};
  v.B = (int)p->batch;
  v.T = (int)p->T;
  v.K = (int)p->K;
  v.C = (int)p->C;
  v.cum = p->cum_scores;
  v.tr = p->transition;
  v.db = p->duration_bias;
  v.ps = p->proj_start;
  v.pe = p->proj_end;
  v.lengths = p->lengths;
  return v;
}

}  // namespace

extern "C" {

int semicrf_abi_version(void) { return SEMICRF_ABI_VERSION; }

const char* semicrf_strerror(int status) {
  switch (status) {
    case SEMICRF_OK: return "ok";
    case SEMICRF_ERR_INVALID_ARGUMENT: return "invalid argument";
    case SEMICRF_ERR_UNSUPPORTED: return "unsupported problem shape";
    case SEMICRF_ERR_WORKSPACE: return "workspace too small";
    case SEMICRF_ERR_CUDA: return "CUDA launch failed";
    case SEMICRF_ERR_SEMIRING: return "semiring must be 'log' or 'max'";
    default: return "unknown error";
  }
}

int64_t semicrf_checkpoint_interval(int64_t T, int64_t K) {
  const int64_t opt = (int64_t)std::sqrt((double)(T * K));
  return opt > K ? opt : K;
}

size_t semicrf_saved_size(const semicrf_problem* p) {
  if (validate_shape(p) != SEMICRF_OK) return 0;
  Carver cv(nullptr);
  carve_saved(cv, p);
  return cv.bytes();
}

size_t semicrf_forward_workspace_size(const semicrf_problem* p) {
  if (validate_shape(p) != SEMICRF_OK) return 0;
  Carver cv(nullptr);
  if (p->transition_ndim == 3)
    carve_kcc(cv, p, false);
  else
    carve_prep(cv, (int)p->C, (int)p->K, p->semiring);
  return cv.bytes();
}

namespace {

// Reference-layout ring checkpoints (triton_forward.py:554-714: checkpoint i
// holds alpha of the K positions ending at i*S, slot p % K; unset entries are
// NEG_INF; checkpoint 0 holds alpha[0] = 0) from the kept float64 alpha tables
// (a = exp(alpha - n)).  The same entries as the generic chain writes when it
// produces them itself: position u >= 1 goes to checkpoint ceil(u / S) if that
// checkpoint lies at or before the sequence end and within K - 1 of u.
__global__ void rings_from_tables_kernel(const double* a_tab, const double* n_tab,
                                         const int64_t* lengths, float* rings, int B, int T,
                                         int K, int C, int nref, int S) {
  const size_t total = (size_t)B * nref * K * C;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const int slot = (int)((i / C) % K);
    const int ic = (int)((i / ((size_t)C * K)) % nref);
    const int b = (int)(i / ((size_t)C * K * nref));
    const long long lraw = lengths[b];
    const int Lb = lraw < 0 ? 0 : (lraw > T ? T : (int)lraw);
    float v = kRefNegInf;
    if (ic == 0) {
      if (slot == 0) v = 0.f;
    } else if ((long long)ic * S <= Lb) {
      // the position of this slot in (ic*S - K, ic*S]
      const int top = ic * S;
      int u = top - ((top - slot) % K + K) % K;
      if (u >= 1 && u > top - K && u > (ic - 1) * S) {
        const size_t row = (size_t)b * (T + 1) + u;
        const double a = a_tab[row * C + c];
        v = a > 0.0 ? (float)(log(a) + n_tab[row]) : kRefNegInf;
      }
    }
    rings[i] = v;
  }
}

cudaError_t launch_rings_from_tables(const semicrf_problem* p, const double* a_tab,
                                     const double* n_tab, float* rings, int nref,
                                     cudaStream_t s) {
  const size_t total = (size_t)p->batch * nref * p->K * p->C;
  if (total == 0) return cudaSuccess;
  int g = (int)((total + 255) / 256);
  if (g > device_sm_count() * 8) g = device_sm_count() * 8;
  rings_from_tables_kernel<<<g, 256, 0, s>>>(a_tab, n_tab, p->lengths, rings, (int)p->batch,
                                             (int)p->T, (int)p->K, (int)p->C, nref,
                                             (int)p->checkpoint_interval);
  return cudaGetLastError();
}

}  // namespace

int semicrf_forward(const semicrf_problem* p, float* partition, float* ring_checkpoints,
                    int64_t num_ring_checkpoints, void* saved, void* workspace,
                    size_t workspace_bytes, void* stream) {
  int st = validate(p);
  if (st != SEMICRF_OK) return st;
  if (p->batch == 0) return SEMICRF_OK;
  if (!partition) return SEMICRF_ERR_INVALID_ARGUMENT;
  if (ring_checkpoints && num_ring_checkpoints < 1) return SEMICRF_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < semicrf_forward_workspace_size(p) || !workspace)
    return SEMICRF_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p->transition_ndim == 3) {
    // (K, C, C): the alpha chain, and beside it the beta chain when a
    // backward will follow (both tables are kept)
    Carver cv(workspace);
    KccLayout w = carve_kcc(cv, p, false);
    cudaError_t e = launch_kcc_prep(p->transition, p->duration_bias, (int)p->K, (int)p->C,
                                    w.pr, s);
    if (e != cudaSuccess) return SEMICRF_ERR_CUDA;
    KccArgs a = kcc_args(p, w.pr);
    a.kflag = w.kflag;
    a.partition = partition;
    a.ref_ckpt = ring_checkpoints;
    a.nref = (int)num_ring_checkpoints;
    a.sref = (int)p->checkpoint_interval;
    if (saved) {
      Carver sc(saved);
      SavedLayout sl = carve_saved(sc, p);
      a.logz = sl.logz;
      a.alpha = sl.a_tab;
      a.amax = sl.n_tab;
      a.beta = sl.b_tab;
    }
    return cuda_status(launch_kcc_chains(a, saved ? 2 : 1, s));
  }
  if (p->semiring == SEMICRF_MAX && !saved && !ring_checkpoints &&
      vchain_supported((int)p->batch, (int)p->C, (int)p->K)) {
    // score only: one warp per sequence, no prepared tables needed
    VChainArgs v = vchain_args(p);
    v.partition = partition;
    return cuda_status(launch_vchain(v, s));
  }
  Carver cv(workspace);
  Prepared pr = carve_prep(cv, (int)p->C, (int)p->K, p->semiring);
  cudaError_t e = launch_prep(p->transition, p->duration_bias, (int)p->K, (int)p->C,
                              kcap_of(p->K), kP, p->semiring, pr, s);
  if (e != cudaSuccess) return SEMICRF_ERR_CUDA;
  if (p->semiring == SEMICRF_LOG) {
    LChainLaunch L{};
    L.B = (int)p->batch;
    L.T = (int)p->T;
    L.K = (int)p->K;
    L.C = (int)p->C;
    L.dbe = pr.dbed;
    L.dbmax = pr.dbmax;
    LChainArgs a{};
    a.mode = 0;
    a.dir = 0;
    a.cum = p->cum_scores;
    a.ps = p->proj_start;
    a.pe = p->proj_end;
    a.lengths = p->lengths;
    a.mx = pr.mxd_f;
    a.colmax = pr.colmax_f;
    a.partition = partition;
    a.ref_ckpt = ring_checkpoints;
    a.nref = (int)num_ring_checkpoints;
    a.sref = (int)p->checkpoint_interval;
    a.sint = sint_of(p);
    a.nint = nint_of(p);
    L.a0 = a;
    L.a1 = a;
    L.n1 = (int)p->batch;
    int grid = (int)p->batch;
    int* rec_ovf = nullptr;
    if (saved && p->backward_mode != SEMICRF_RECOMPUTE && ring_checkpoints) {
      // keep mode with the reference-layout checkpoints: the chains run as
      // without them (whole or time-chunked, warp-specialised or clustered)
      // and the checkpoints are then read off the kept alpha tables
      semicrf_problem q = *p;
      const int st = semicrf_forward(&q, partition, nullptr, 0, saved, workspace,
                                     workspace_bytes, stream);
      if (st != SEMICRF_OK) return st;
      Carver sc(saved);
      SavedLayout sl = carve_saved(sc, p);
      return cuda_status(launch_rings_from_tables(p, sl.a_tab, sl.n_tab, ring_checkpoints,
                                                  (int)num_ring_checkpoints, s));
    }
    if (saved) {
      Carver sc(saved);
      SavedLayout sl = carve_saved(sc, p);
      L.a0.logz = sl.logz;
      if (p->backward_mode == SEMICRF_RECOMPUTE) {
        L.a0.sv = sl.sv;
        L.a0.write_saved = 1;
        rec_ovf = sl.rec_ovf;
      } else {
        // keep both chains' tables: the beta chain does not depend on alpha,
        // so it runs beside the alpha chain in the same launch
        L.a0.a_tab = sl.a_tab;
        L.a0.A_tab = sl.A_tab;
        L.a0.n_tab = sl.n_tab;
        L.a1 = beta_chain_args(p, pr, sl.b_tab, sl.B_tab, sl.m_tab);
        grid = 2 * (int)p->batch;
        if (sl.cp.nchunk > 1 && !L.a0.ref_ckpt) {
          // as below: a log-domain rerun of whole chains when a chunk's frames clip
          const bool fix = lchain_fix_supported((int)p->C, (int)p->K);
          if (fix) {
            L.dbl = pr.dbl;
            L.ovf = pr.ovf;
            if (cudaMemsetAsync(pr.ovf, 0, sizeof(int), s) != cudaSuccess)
              return SEMICRF_ERR_CUDA;
          }
          cudaError_t e2 = chunked_chains(p, L, sl, s);
          if (e2 != cudaSuccess || !fix) return cuda_status(e2);
          return cuda_status(launch_lchain_fix(L, grid, s));
        }
      }
    }
    if (!L.a0.ref_ckpt && !L.a0.write_saved && lchain_ws_supported((int)p->C, (int)p->K)) {
      // the log-domain rerun when the chain's float64 frames clip (extreme scores)
      const bool fix = lchain_fix_supported((int)p->C, (int)p->K);
      if (fix) {
        L.dbl = pr.dbl;
        L.ovf = pr.ovf;
        if (cudaMemsetAsync(pr.ovf, 0, sizeof(int), s) != cudaSuccess) return SEMICRF_ERR_CUDA;
      }
      cudaError_t e2 = launch_lchain_ws(L, grid, s);
      if (e2 != cudaSuccess || !fix) return cuda_status(e2);
      return cuda_status(launch_lchain_fix(L, grid, s));
    }
    if (!L.a0.ref_ckpt && !L.a0.write_saved && lchain_cl_supported((int)p->C, (int)p->K)) {
      // the same log-domain rerun for the cluster chain (64 < C <= 256)
      const bool fix = lchain_fix_supported((int)p->C, (int)p->K);
      if (fix) {
        L.dbl = pr.dbl;
        L.ovf = pr.ovf;
        if (cudaMemsetAsync(pr.ovf, 0, sizeof(int), s) != cudaSuccess) return SEMICRF_ERR_CUDA;
      }
      cudaError_t e2 = launch_lchain_cl(L, grid, s);
      if (e2 != cudaSuccess || !fix) return cuda_status(e2);
      return cuda_status(launch_lchain_fix(L, grid, s));
    }
    // the generic chain: the same rerun for whole chains (ring checkpoints
    // included).  In the recompute mode the flag lives in the saved state: the
    // rerun corrects log Z and the partition here, and the backward, finding
    // the flag set, rebuilds its tables in the log domain instead of from the
    // (clipped) restart records.
    const bool fix = lchain_fix_supported((int)p->C, (int)p->K);
    int* ovf = rec_ovf ? rec_ovf : pr.ovf;
    if (fix || rec_ovf) {
      L.dbl = pr.dbl;
      L.ovf = ovf;
      if (cudaMemsetAsync(ovf, 0, sizeof(int), s) != cudaSuccess) return SEMICRF_ERR_CUDA;
    }
    cudaError_t e2 = launch_lchain(L, grid, s);
    if (e2 != cudaSuccess || !fix) return cuda_status(e2);
    return cuda_status(launch_lchain_fix(L, grid, s));
  }
  ChainLaunch L = base_launch(p, pr);
  ChainArgs a = base_args(p);
  a.mode = 0;
  a.dir = 0;
  a.mx = pr.mx_f;
  a.colmax = pr.colmax_f;
  a.partition = partition;
  a.ref_ckpt = ring_checkpoints;
  a.nref = (int)num_ring_checkpoints;
  a.sref = (int)p->checkpoint_interval;
  a.sint = sint_of(p);
  a.nint = nint_of(p);
  if (saved) {
    Carver sc(saved);
    SavedLayout sl = carve_saved(sc, p);
    a.logz = sl.logz;
    a.sv_f = sl.sv_f;
    a.sv_d = sl.sv_d;
    a.write_saved = 1;
  }
  L.a0 = a;
  L.a1 = a;
  L.n1 = (int)p->batch;
  return cuda_status(launch_chain(L, (int)p->batch, p->semiring, false, s));
}

size_t semicrf_backward_workspace_size(const semicrf_problem* p) {
  if (validate_shape(p) != SEMICRF_OK) return 0;
  Carver cv(nullptr);
  if (p->transition_ndim == 3)
    carve_kcc(cv, p, true);
  else if (p->semiring == SEMICRF_LOG)
    carve_lbwd(cv, p);
  else
    carve_bwd(cv, p);
  return cv.bytes();
}

int semicrf_backward(const semicrf_problem* p, const void* saved, const float* grad_output,
                     float* grad_cum, float* grad_transition, float* grad_duration_bias,
                     float* grad_proj_start, float* grad_proj_end, void* workspace,
                     size_t workspace_bytes, void* stream) {
  int st = validate(p);
  if (st != SEMICRF_OK) return st;
  if (p->batch == 0) return SEMICRF_OK;
  if (!saved || !grad_output || !grad_cum || !grad_transition || !grad_duration_bias)
    return SEMICRF_ERR_INVALID_ARGUMENT;
  if ((p->proj_start && !grad_proj_start) || (p->proj_end && !grad_proj_end))
    return SEMICRF_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < semicrf_backward_workspace_size(p) || !workspace)
    return SEMICRF_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p->transition_ndim == 3) {
    Carver cv(workspace);
    KccLayout w = carve_kcc(cv, p, true);
    Carver sc(const_cast<void*>(saved));
    SavedLayout sl = carve_saved(sc, p);
    cudaError_t e = launch_kcc_prep(p->transition, p->duration_bias, (int)p->K, (int)p->C,
                                    w.pr, s);
    if (e != cudaSuccess) return SEMICRF_ERR_CUDA;
    KccArgs a = kcc_args(p, w.pr);
    a.logz = sl.logz;
    a.alpha = sl.a_tab;
    a.amax = sl.n_tab;
    a.beta = sl.b_tab;
    a.grad_output = grad_output;
    a.grad_cum = grad_cum;
    a.grad_ps = p->proj_start ? grad_proj_start : nullptr;
    a.grad_pe = p->proj_end ? grad_proj_end : nullptr;
    a.st = w.st;
    a.et = w.et;
    a.pend = w.pend;
    a.part_tr = w.part_tr;
    a.nslice = w.nslice;
    a.al = w.al;
    a.anc = w.anc;
    a.ep1 = w.ep1;
    a.kflag = w.kflag;
    return cuda_status(launch_kcc_grads(a, grad_transition, grad_duration_bias, s));
  }
  if (p->semiring == SEMICRF_LOG) {
    Carver cv(workspace);
    LBwdLayout w = carve_lbwd(cv, p);
    Carver sc(const_cast<void*>(saved));
    SavedLayout sl = carve_saved(sc, p);
    cudaError_t e = cudaSuccess;
    LChainLaunch L{};
    L.B = (int)p->batch;
    L.T = (int)p->T;
    L.K = (int)p->K;
    L.C = (int)p->C;
    L.dbe = w.pr.dbed;
    L.dbmax = w.pr.dbmax;
    const double *xa = sl.a_tab, *xA = sl.A_tab, *xn = sl.n_tab;
    const double *ya = sl.b_tab, *yA = sl.B_tab, *yn = sl.m_tab;
    if (p->backward_mode == SEMICRF_RECOMPUTE) {
      // alpha between checkpoints (all segments of all sequences in parallel)
      // and the beta chains
      e = launch_prep(p->transition, p->duration_bias, (int)p->K, (int)p->C, kcap_of(p->K), kP,
                      SEMICRF_LOG, w.pr, s);
      if (e != cudaSuccess) return SEMICRF_ERR_CUDA;
      LChainArgs r{};
      r.mode = 1;
      r.dir = 0;
      r.cum = p->cum_scores;
      r.ps = p->proj_start;
      r.pe = p->proj_end;
      r.lengths = p->lengths;
      r.mx = w.pr.mxd_f;
      r.colmax = w.pr.colmax_f;
      r.sv = sl.sv;
      r.sint = sint_of(p);
      r.nint = nint_of(p);
      r.a_tab = w.a_tab;
      r.A_tab = w.A_tab;
      r.n_tab = w.n_tab;
      const LChainArgs bb = beta_chain_args(p, w.pr, w.b_tab, w.B_tab, w.m_tab);
      if (lchain_fix_supported((int)p->C, (int)p->K)) {
        // start from the forward's flag; the launches below may set it too
        L.dbl = w.pr.dbl;
        L.ovf = w.pr.ovf;
        if (cudaMemcpyAsync(w.pr.ovf, sl.rec_ovf, sizeof(int), cudaMemcpyDeviceToDevice, s) !=
            cudaSuccess)
          return SEMICRF_ERR_CUDA;
      }
      L.a0 = r;
      L.n1 = (int)p->batch * r.nint;
      if (lchain_ws_supported((int)p->C, (int)p->K)) {
        L.a1 = r;
        e = launch_lchain(L, L.n1, s);
        if (e != cudaSuccess) return SEMICRF_ERR_CUDA;
        LChainLaunch Lb = L;
        Lb.a0 = bb;
        Lb.a1 = bb;
        Lb.n1 = (int)p->batch;
        e = launch_lchain_ws(Lb, (int)p->batch, s);
      } else {
        L.a1 = bb;
        e = launch_lchain(L, L.n1 + (int)p->batch, s);
      }
      if (e != cudaSuccess) return SEMICRF_ERR_CUDA;
      if (lchain_fix_supported((int)p->C, (int)p->K)) {
        // frames that clipped, in the forward (its flag, saved) or in the
        // recompute above: both chains again, whole, in the log domain,
        // rewriting the tables (log Z is the forward's, already corrected)
        LChainLaunch Lf = L;
        Lf.a0 = r;
        Lf.a0.mode = 0;
        Lf.a0.sv = nullptr;
        Lf.a1 = bb;
        Lf.n1 = (int)p->batch;
        e = launch_lchain_fix(Lf, 2 * (int)p->batch, s);
        if (e != cudaSuccess) return SEMICRF_ERR_CUDA;
      }
      xa = w.a_tab;
      xA = w.A_tab;
      xn = w.n_tab;
      ya = w.b_tab;
      yA = w.B_tab;
      yn = w.m_tab;
    }
    LMargArgs m{};
    m.B = (int)p->batch;
    m.T = (int)p->T;
    m.K = (int)p->K;
    m.C = (int)p->C;
    m.kcap = kcap_of(p->K);
    m.cum = p->cum_scores;
    m.ps = p->proj_start;
    m.pe = p->proj_end;
    m.tr = p->transition;
    m.db = p->duration_bias;
    m.lengths = p->lengths;
    m.logz = sl.logz;
    m.grad_output = grad_output;
    m.xa = xa;
    m.xA = xA;
    m.xn = xn;
    m.ya = ya;
    m.yA = yA;
    m.yn = yn;
    m.grad_cum = grad_cum;
    m.grad_ps = p->proj_start ? grad_proj_start : nullptr;
    m.grad_pe = p->proj_end ? grad_proj_end : nullptr;
    m.la = w.la;
    m.lb = w.lb;
    m.maX = w.maX;
    m.mbY = w.mbY;
    m.part_tr = w.part_tr;
    m.nchunk = w.mp.nchunk;
    m.part_db = w.part_db;
    m.nsplit = w.mp.nsplit;
    m.cg = w.mp.cg;
    m.dbflag = w.dbflag;
    return cuda_status(launch_lmarg(m, grad_transition, grad_duration_bias, s));
  }
  Carver cv(workspace);
  BwdLayout w = carve_bwd(cv, p);
  Carver sc(const_cast<void*>(saved));
  SavedLayout sl = carve_saved(sc, p);
  cudaError_t e = launch_prep(p->transition, p->duration_bias, (int)p->K, (int)p->C,
                              kcap_of(p->K), kP, p->semiring, w.pr, s);
  if (e != cudaSuccess) return SEMICRF_ERR_CUDA;

  // beta chains (one per sequence) and alpha checkpoint segments, one launch
  ChainLaunch L = base_launch(p, w.pr);
  ChainArgs ab = base_args(p);
  ab.mode = 0;
  ab.dir = 1;
  ab.mx = w.pr.mx_b;
  ab.colmax = w.pr.colmax_b;
  ab.tab_x = w.xb;
  ab.tab_m = w.mb;
  ab.tab_n = w.nb;
  ChainArgs aa = base_args(p);
  aa.mode = 1;
  aa.dir = 0;
  aa.mx = w.pr.mx_f;
  aa.colmax = w.pr.colmax_f;
  aa.sv_f = sl.sv_f;
  aa.sv_d = sl.sv_d;
  aa.sint = sint_of(p);
  aa.nint = nint_of(p);
  aa.tab_x = w.xa;
  aa.tab_m = w.ma;
  aa.tab_n = w.na;
  L.a0 = ab;
  L.a1 = aa;
  L.n1 = (int)p->batch;
  const int grid = (int)p->batch + (int)p->batch * aa.nint;
  e = launch_chain(L, grid, p->semiring, false, s);
  if (e != cudaSuccess) return SEMICRF_ERR_CUDA;

  MargArgs m{};
  m.B = (int)p->batch;
  m.T = (int)p->T;
  m.K = (int)p->K;
  m.C = (int)p->C;
  m.kcap = kcap_of(p->K);
  m.cum = p->cum_scores;
  m.ps = p->proj_start;
  m.pe = p->proj_end;
  m.tr = p->transition;
  m.dbl = w.pr.dbl;
  m.lengths = p->lengths;
  m.logz = sl.logz;
  m.grad_output = grad_output;
  m.xa = w.xa;
  m.ma = w.ma;
  m.na = w.na;
  m.xb = w.xb;
  m.mb = w.mb;
  m.nb = w.nb;
  m.grad_cum = grad_cum;
  m.grad_ps = p->proj_start ? grad_proj_start : nullptr;
  m.grad_pe = p->proj_end ? grad_proj_end : nullptr;
  m.part_tr = w.part_tr;
  m.part_db = w.part_db;
  e = launch_marginals_impl(m, p->semiring, w.alse, w.pstart, s);
  if (e != cudaSuccess) return SEMICRF_ERR_CUDA;
  return cuda_status(launch_reduce_shared(m, grad_transition, grad_duration_bias, s));
}

size_t semicrf_viterbi_workspace_size(const semicrf_problem* p) {
  if (validate_shape(p) != SEMICRF_OK || p->transition_ndim != 2) return 0;
  Carver cv(nullptr);
  carve_vit(cv, p);
  return cv.bytes();
}

int semicrf_viterbi(const semicrf_problem* p, int64_t max_traceback_length, float* scores,
                    int32_t* seg_start, int32_t* seg_end, int32_t* seg_label, double* seg_score,
                    int32_t* nseg, void* workspace, size_t workspace_bytes, void* stream) {
  int st = validate(p);
  if (st != SEMICRF_OK) return st;
  if (p->transition_ndim != 2) return SEMICRF_ERR_UNSUPPORTED;  // nn.py:460 takes (C, C)
  if (p->batch == 0) return SEMICRF_OK;
  if (p->semiring != SEMICRF_MAX) return SEMICRF_ERR_SEMIRING;
  if (p->proj_start || p->proj_end) return SEMICRF_ERR_UNSUPPORTED;  // nn.py:479 has none
  if (!scores || !seg_start || !seg_end || !seg_label || !seg_score || !nseg)
    return SEMICRF_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < semicrf_viterbi_workspace_size(p) || !workspace)
    return SEMICRF_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Carver cv(workspace);
  VitLayout w = carve_vit(cv, p);
  cudaError_t e;
  if (vchain_supported((int)p->batch, (int)p->C, (int)p->K)) {
    // warp chain; the backtrace walks packed backpointers staged in shared
    // memory when one sequence's fit, else the separate arrays in global memory
    const bool packed = p->T <= 32767 && backtrace_packed_smem((int)p->T, (int)p->C) <= 200 * 1024;
    VChainArgs v = vchain_args(p);
    v.partition = scores;
    v.final_c = w.final_c;
    if (packed) {
      v.bp = w.bp;
    } else {
      v.bp_k = w.bp_k;
      v.bp_c = w.bp_c;
    }
    e = launch_vchain(v, s);
    if (e != cudaSuccess) return SEMICRF_ERR_CUDA;
    if (packed)
      return cuda_status(launch_backtrace_packed(
          (int)p->batch, (int)p->T, (int)p->K, (int)p->C, p->cum_scores, p->transition,
          p->duration_bias, p->lengths, max_traceback_length, w.bp, w.final_c, seg_start, seg_end,
          seg_label, seg_score, nseg, s));
    return cuda_status(launch_backtrace((int)p->batch, (int)p->T, (int)p->K, (int)p->C,
                                        p->cum_scores, p->transition, p->duration_bias,
                                        p->lengths, max_traceback_length, w.bp_k, w.bp_c,
                                        w.final_c, seg_start, seg_end, seg_label, seg_score,
                                        nseg, s));
  }
  e = launch_prep(p->transition, p->duration_bias, (int)p->K, (int)p->C, kcap_of(p->K), kP,
                  SEMICRF_MAX, w.pr, s);
  if (e != cudaSuccess) return SEMICRF_ERR_CUDA;
  ChainLaunch L = base_launch(p, w.pr);
  ChainArgs a = base_args(p);
  a.mode = 0;
  a.dir = 0;
  a.mx = w.pr.mx_f;
  a.colmax = w.pr.colmax_f;
  a.score = scores;
  a.bp_k = w.bp_k;
  a.bp_c = w.bp_c;
  a.final_c = w.final_c;
  L.a0 = a;
  L.a1 = a;
  L.n1 = (int)p->batch;
  e = launch_chain(L, (int)p->batch, SEMICRF_MAX, true, s);
  if (e != cudaSuccess) return SEMICRF_ERR_CUDA;
  return cuda_status(launch_backtrace((int)p->batch, (int)p->T, (int)p->K, (int)p->C,
                                      p->cum_scores, p->transition, p->duration_bias,
                                      p->lengths, max_traceback_length, w.bp_k, w.bp_c,
                                      w.final_c, seg_start, seg_end, seg_label, seg_score,
                                      nseg, s));
}

int semicrf_score_gold(int64_t B, int64_t T, int64_t K, int64_t C, const float* cum_scores,
                       const int64_t* labels, const int64_t* lengths, const float* transition,
                       const float* duration_bias, float* out, void* stream) {
  if (B < 0 || T < 0 || K < 1 || C < 1) return SEMICRF_ERR_INVALID_ARGUMENT;
  if (B == 0) return SEMICRF_OK;
  if (T == 1 && K < 2) return SEMICRF_ERR_INVALID_ARGUMENT;  // helpers.py:412 indexes db[1]
  if (!cum_scores || !labels || !lengths || !transition || !duration_bias || !out)
    return SEMICRF_ERR_INVALID_ARGUMENT;
  return cuda_status(launch_gold((int)B, (int)T, (int)K, (int)C, cum_scores, labels, lengths,
                                 transition, duration_bias, out,
                                 static_cast<cudaStream_t>(stream)));
}

size_t semicrf_score_gold_workspace_size(int64_t B, int64_t T, int64_t K, int64_t C) {
  (void)T;
  if (B < 0 || K < 1 || C < 1) return 0;
  return (size_t)B * (C * C + K * C) * sizeof(float) + 256;
}

int semicrf_score_gold_backward(int64_t B, int64_t T, int64_t K, int64_t C,
                                const int64_t* labels, const int64_t* lengths,
                                const float* grad_out, float* grad_cum, float* grad_transition,
                                float* grad_duration_bias, void* workspace,
                                size_t workspace_bytes, void* stream) {
  if (B < 0 || T < 0 || K < 1 || C < 1) return SEMICRF_ERR_INVALID_ARGUMENT;
  if (T == 1 && K < 2) return SEMICRF_ERR_INVALID_ARGUMENT;
  if (B == 0) return SEMICRF_OK;
  if (!labels || !lengths || !grad_out || !grad_cum || !grad_transition || !grad_duration_bias)
    return SEMICRF_ERR_INVALID_ARGUMENT;
  if (!workspace || workspace_bytes < semicrf_score_gold_workspace_size(B, T, K, C))
    return SEMICRF_ERR_WORKSPACE;
  return cuda_status(launch_gold_backward((int)B, (int)T, (int)K, (int)C, labels, lengths,
                                          grad_out, grad_cum, grad_transition,
                                          grad_duration_bias, static_cast<float*>(workspace),
                                          static_cast<cudaStream_t>(stream)));
}

}  // extern "C"

// ---- edge-tensor scan --------------------------------------------------------

namespace {

int es_validate(int64_t B, int64_t N, int64_t K, int64_t C, int semiring) {
  if (B < 0 || N < 1 || K < 1 || C < 1) return SEMICRF_ERR_INVALID_ARGUMENT;
  if (semiring != SEMICRF_LOG && semiring != SEMICRF_MAX) return SEMICRF_ERR_SEMIRING;
  if (N > (int64_t)1 << 30 || K > 32767 || C > 32767 || !escan_supported((int)K, (int)C))
    return SEMICRF_ERR_UNSUPPORTED;
  return SEMICRF_OK;
}

struct EsSaved {
  double *logz, *beta;
  int32_t* bp;
};

EsSaved es_carve(Carver& cv, int64_t B, int64_t N, int64_t C, int semiring) {
  EsSaved e{};
  e.logz = cv.take<double>(B);
  e.beta = cv.take<double>((size_t)B * N * C);
  e.bp = semiring == SEMICRF_MAX ? cv.take<int32_t>((size_t)B * N * C) : nullptr;
  return e;
}

}  // namespace

extern "C" {

size_t semicrf_edge_scan_saved_size(int64_t B, int64_t N, int64_t K, int64_t C, int semiring) {
  if (es_validate(B, N, K, C, semiring) != SEMICRF_OK) return 0;
  Carver cv(nullptr);
  es_carve(cv, B, N, C, semiring);
  return cv.bytes();
}

int semicrf_edge_scan_forward(int64_t B, int64_t N, int64_t K, int64_t C, const float* edge,
                              const int64_t* lengths, int semiring, float* partition, void* saved,
                              void* stream) {
  int st = es_validate(B, N, K, C, semiring);
  if (st != SEMICRF_OK) return st;
  if (B == 0) return SEMICRF_OK;
  if (!lengths || !partition || (N > 1 && !edge)) return SEMICRF_ERR_INVALID_ARGUMENT;
  EsSaved e{};
  if (saved) {
    Carver cv(saved);
    e = es_carve(cv, B, N, C, semiring);
  }
  return cuda_status(launch_escan_forward((int)B, (int)N, (int)K, (int)C, edge, lengths, semiring,
                                          partition, e.logz, e.beta, e.bp,
                                          static_cast<cudaStream_t>(stream)));
}

size_t semicrf_edge_scan_backward_workspace_size(int64_t B, int64_t N, int64_t K, int64_t C,
                                                 int semiring) {
  if (es_validate(B, N, K, C, semiring) != SEMICRF_OK) return 0;
  Carver cv(nullptr);
  if (semiring == SEMICRF_LOG) cv.take<double>((size_t)B * N * C);
  return cv.bytes() > 0 ? cv.bytes() : 256;
}

int semicrf_edge_scan_backward(int64_t B, int64_t N, int64_t K, int64_t C, const float* edge,
                               const int64_t* lengths, int semiring, const void* saved,
                               const float* grad_out, float* grad_edge, void* workspace,
                               size_t workspace_bytes, void* stream) {
  int st = es_validate(B, N, K, C, semiring);
  if (st != SEMICRF_OK) return st;
  if (B == 0 || N == 1) return SEMICRF_OK;  // no edges
  if (!edge || !lengths || !saved || !grad_out || !grad_edge) return SEMICRF_ERR_INVALID_ARGUMENT;
  if (!workspace || workspace_bytes < semicrf_edge_scan_backward_workspace_size(B, N, K, C, semiring))
    return SEMICRF_ERR_WORKSPACE;
  Carver sc(const_cast<void*>(saved));
  const EsSaved e = es_carve(sc, B, N, C, semiring);
  Carver cv(workspace);
  double* gamma = semiring == SEMICRF_LOG ? cv.take<double>((size_t)B * N * C) : nullptr;
  return cuda_status(launch_escan_backward((int)B, (int)N, (int)K, (int)C, edge, lengths,
                                           semiring, e.beta, e.logz, e.bp, grad_out, grad_edge,
                                           gamma, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
