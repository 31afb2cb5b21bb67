// lchain_ws.cu -- warp-specialised float64 log-semiring chain (C <= 64).
//
// Same recurrence and linear-domain float64 formulation as lchain.cu (see
// there for the derivation and the reference citations), reorganised so that
// the per-position critical path never waits for bulk work:
//
//   serial warp(s)  (one lane per label): for block tau of LP targets, the
//       near sources (blocks tau-1 and tau), the state a, the float64 mat-vec
//       and the new source E.  About a dozen dependent float64 operations
//       plus one shared-memory broadcast per position.
//   bulk warps      (the other warps but the idle ones): while the serial
//       warp works on block tau they prepare block tau+1 -- its normaliser,
//       frame factors, g/h factors and the far part of every target's k-sum
//       (all sources before block tau).
// The same kernel runs the alpha chain (dir = 0) and the beta chain (dir = 1,
// the recurrence reversed); both write their float64 tables, from which
// lmarg.cu derives the gradients.
// Hand-off uses named barriers (FULL[b]: bulk -> serial, DONE[b]: serial ->
// bulk, double-buffered by block parity).
//
// Frames.  Each block beta has a normaliser n_beta and a per-label content
// anchor cA_beta[c] = cum(u0_beta, c).  Sources of block beta are stored as
//     E[s,c] = exp(m[s,c] + soff(s,c) - n_beta - csign*(cum(s,c) - cA_beta[c]))
// and enter the k-sum of a target in block tau with the factor
//     W[beta->tau,c] = prod_{gamma=beta}^{tau-1} w_gamma[c],
//     w_gamma[c]    = exp(n_gamma - n_{gamma+1} + csign*(cA_{gamma+1}[c] - cA_gamma[c])).
// Targets use a[u,c] = g[u,c] * sum_s E[s,c] W Db[u-s,c] with
//     g[u,c] = exp(toff(u,c) + dbmax[c] + csign*(cum(u,c) - cA_tau[c])),
// and new sources E[u,c] = ym[u,c] * h[u,c],
//     h[u,c] = exp(colmax[c] + soff(u,c) - csign*(cum(u,c) - cA_tau[c])).
// Nothing in the ring is ever rewritten, so the bulk warps can read it while
// the serial warp appends.  n_tau is predicted two blocks ahead from the
// measured scale of the state (float64 leaves a very wide margin for the
// prediction error).

#include <type_traits>

#include "semicrf_internal.cuh"

namespace semicrf {

#ifdef SEMICRF_TIMING
__device__ unsigned long long g_wstim[256][16];
#define WT_DECL unsigned long long wt_[16] = {}; unsigned long long wck_ = clock64();
#define WT_ADD(i) (wt_[i] += clock64() - wck_, wck_ = clock64())
#define WT_FLUSH(lo)                                                              \
  if ((tid == 0 || tid == CP) && blockIdx.x < 256)                                  \
    for (int q_ = 0; q_ < 8; ++q_) g_wstim[blockIdx.x][(lo) + q_] = wt_[(lo) + q_];
#else
#define WT_DECL
#define WT_ADD(i)
#define WT_FLUSH(lo)
#endif

namespace {

constexpr int kWsThreads = 256;  // 2 warps per SM sub-partition
constexpr size_t kWsSmemMax = 227 * 1024;

enum : int { kBarFull0 = 1, kBarFull1 = 2, kBarDone0 = 3, kBarDone1 = 4, kBarBulk = 5,
             kBarSerial = 6 };

__device__ __forceinline__ void bar_arrive(int id, int n) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

struct WsPlan {
  int C, Cs, CP, K, kcap, LP, R, NR, kx, nbr, nbulk, np, nsplit, nwt;
  int nsplit1, bpc1;  // single-label far-sum items: splits per label, source blocks per split
  int o_ring, o_dbd, o_mx, o_dbmax, o_colmax, o_nring, o_ca, o_da, o_far, o_g,
      o_h, o_wprev, o_part, o_abuf, o_wt, o_misc, o_edb, o_ecm, o_alast;
  int bytes;
};

// Shared-memory layout.  The source ring has R = NR*LP slots (at least
// kcap + 2*LP) of Cs = C rounded up to even labels: position u lives in slot
// (u - 1) mod R, so every block of LP sources occupies LP consecutive slots
// and a label pair is one 16-byte load.
__host__ __device__ inline void ws_make(WsPlan& p, int C, int K, int CP, int LP) {
  p.C = C;
  p.Cs = C + (C & 1);
  p.CP = CP;
  p.K = K;
  p.kcap = K > 1 ? K - 1 : 1;
  p.LP = LP;
  p.NR = (p.kcap + 2 * LP + LP - 1) / LP;
  p.R = p.NR * LP;
  p.kx = p.kcap + kPrepRowsExtra;
  int nbr = p.NR + 4;  // blocks whose frame factors are kept (power of 2)
  p.nbr = 1;
  while (p.nbr < nbr) p.nbr <<= 1;
  // every warp on a sub-partition that hosts a serial warp idles
  p.nbulk = kWsThreads - (kWsThreads / 128) * CP;
  p.np = p.Cs / 2;
  p.nsplit = p.nbulk / p.np > 0 ? p.nbulk / p.np : 1;
  // single-label items (label, split): each covers bpc1 consecutive source
  // blocks of the at most ceil(kcap / LP) - 1 a target block reaches
  p.nsplit1 = p.nbulk / C > 0 ? p.nbulk / C : 1;
  const int nq_max = (p.kcap + LP - 1) / LP - 1;
  p.bpc1 = nq_max > 0 ? (nq_max + p.nsplit1 - 1) / p.nsplit1 : 0;
  p.nwt = (p.kcap + LP - 1) / LP + 4;  // source blocks a k-window reaches, plus margin
  int o = 0;
  auto take = [&](int n) {
    const int r = o;
    o += (n + 15) & ~15;
    return r;
  };
  p.o_ring = take(8 * p.R * p.Cs);
  p.o_dbd = take(8 * p.kx * p.Cs);  // Db = exp(db - dbmax) as doubles
  p.o_mx = take(8 * C * C);
  p.o_dbmax = take(8 * CP);
  p.o_colmax = take(8 * CP);
  p.o_nring = take(8 * (p.nbr + 2));
  p.o_ca = take(8 * 4 * CP);      // anchors cA of the last four blocks (slot tau mod 4)
  p.o_da = take(8 * 2 * 4 * CP);  // [exp | raw] anchor change csign*(cA_tau - cA_tau-1)
  p.o_far = take(8 * 2 * LP * CP);
  p.o_g = take(8 * 4 * LP * CP);  // g and h of the last four blocks (slot tau mod 4)
  p.o_h = take(8 * 4 * LP * CP);
  p.o_wprev = take(8 * 2 * CP);
  p.o_part = take(8 * p.nsplit * LP * p.Cs);
  p.o_abuf = take(8 * 2 * CP);  // two exchange buffers (alternating positions)
  p.o_wt = take(8 * 2 * p.nwt * p.Cs);  // W tables of the last two prepared blocks
  p.o_misc = take(8 * 16);
  p.o_edb = take(8 * CP);
  p.o_ecm = take(8 * CP);
  p.o_alast = take(8 * 2 * CP);  // the state at the end of the last two blocks
  p.bytes = o;
}

__host__ __device__ inline int ws_cp(int C) { return C <= 32 ? 32 : 64; }

__host__ __device__ inline bool ws_choose(WsPlan& p, int C, int K) {
  if (C > 64) return false;
  ws_make(p, C, K, ws_cp(C), 8);
  return (size_t)p.bytes <= kWsSmemMax;
}

}  // namespace

bool lchain_ws_supported(int C, int K) {
  WsPlan p;
  return ws_choose(p, C, K);
}

// ---------------------------------------------------------------------------
// BPC > 0: the far sums run as single-label items whose duration-bias lags
// stay in registers for the whole chain (BPC source blocks per item, at least
// pl.bpc1); BPC = 0: label-pair items reading the lags from shared memory.
template <int CP, int LP, int BPC>
__global__ void __launch_bounds__(kWsThreads, 1)
    lchain_ws_kernel(const __grid_constant__ LChainLaunch L) {
  extern __shared__ __align__(16) unsigned char smraw[];
  constexpr int SW = CP / 32;
  constexpr int NT = kWsThreads;
  // Warps w and w+4 share a sub-partition.  The serial warps are 0..SW-1;
  // warps 4..4+SW-1 stay idle so that nothing competes with the critical path.
  constexpr int NBT = NT - (NT / 128) * CP;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool serial = tid < CP;
  // warp w runs on sub-partition w % 4: the serial warps' sub-partitions
  // carry nothing else
  const bool idle = !serial && (warp & 3) < SW;
  const int btid = ((warp >> 2) * (4 - SW) + ((warp & 3) - SW)) * 32 + lane;  // bulk index
  constexpr int NPART = CP + NBT;  // threads taking part in FULL / DONE (serial + bulk)
  // CTAs [0, n1) take role a0, the rest role a1 (e.g. the alpha and beta
  // chains of the same batch in one launch)
  const bool role1 = (int)blockIdx.x >= L.n1;
  const LChainArgs& A = role1 ? L.a1 : L.a0;
  const int cta = role1 ? (int)blockIdx.x - L.n1 : (int)blockIdx.x;
  const int nch = A.nchunk > 1 ? A.nchunk : 1;
  const int b = cta / nch, jc = cta % nch;  // sequence and time chunk
  if (b >= L.B) return;
  if (A.only && !A.only[b]) return;
  const int C = L.C, K = L.K, T = L.T;
  const int dir = A.dir;
  const double csign = dir == 0 ? 1.0 : -1.0;
  const long long lraw = A.lengths[b];
  const int Lb = lraw < 0 ? 0 : (lraw > T ? T : (int)lraw);
  // chunk jc > 0 starts A.warm positions before its first output position
  // u_out + 1, from a uniform state (the warm-up); chunk 0 is the exact start
  const int u_out = jc > 0 ? jc * A.chunk_len : -1;
  if (jc > 0 && u_out >= Lb) return;  // nothing of this sequence left
  const int u_begin = jc > 0 ? u_out - A.warm : 0;
  const int u_end = (jc + 1 < nch && (jc + 1) * A.chunk_len < Lb) ? (jc + 1) * A.chunk_len : Lb;
  const int NB = (u_end - u_begin + LP - 1) / LP;  // target blocks

  WsPlan pl;
  ws_choose(pl, C, K);
  const int kcap = pl.kcap, R = pl.R, NR = pl.NR, NBR = pl.nbr, Cs = pl.Cs;
  // which side reduces the block-end state to a scale (the one with slack)
  const bool serial_scale = kcap >= 64;
  double* ring = reinterpret_cast<double*>(smraw + pl.o_ring);  // [R][Cs]
  double* dbd = reinterpret_cast<double*>(smraw + pl.o_dbd);    // [kx][Cs]
  double* mx = reinterpret_cast<double*>(smraw + pl.o_mx);
  double* dbmax = reinterpret_cast<double*>(smraw + pl.o_dbmax);
  double* colmax = reinterpret_cast<double*>(smraw + pl.o_colmax);
  double* nring = reinterpret_cast<double*>(smraw + pl.o_nring);  // n_gamma
  double* cA = reinterpret_cast<double*>(smraw + pl.o_ca);        // [4][CP] anchors (bulk)
  double* dae = reinterpret_cast<double*>(smraw + pl.o_da);       // [4][CP] exp(anchor change)
  double* dar = dae + 4 * CP;                                      // [4][CP] anchor change
  double* farb = reinterpret_cast<double*>(smraw + pl.o_far);     // [2][LP][CP]
  double* gb = reinterpret_cast<double*>(smraw + pl.o_g);
  double* hb = reinterpret_cast<double*>(smraw + pl.o_h);
  double* wprev = reinterpret_cast<double*>(smraw + pl.o_wprev);  // [2][CP]
  double* part = reinterpret_cast<double*>(smraw + pl.o_part);
  double* abuf = reinterpret_cast<double*>(smraw + pl.o_abuf);
  // wt[(tau&1)][q][c] = W[(tau-q) -> tau, c]  (q = 0 .. nwt-1, 0 beyond the start)
  double* wt = reinterpret_cast<double*>(smraw + pl.o_wt);
  const int NWT = pl.nwt;
  double* misc = reinterpret_cast<double*>(smraw + pl.o_misc);
  double* edb = reinterpret_cast<double*>(smraw + pl.o_edb);  // exp(dbmax)
  double* ecm = reinterpret_cast<double*>(smraw + pl.o_ecm);  // exp(colmax)
  double* alast = reinterpret_cast<double*>(smraw + pl.o_alast);  // [2 blocks][CP]
  auto lidx = [&](int gamma) { return (gamma + NBR) & (NBR - 1); };  // gamma >= -NBR

  const float* cum_b = A.cum + (size_t)b * (T + 1) * C;
  const float* ps_b = A.ps ? A.ps + (size_t)b * T * C : nullptr;
  const float* pe_b = A.pe ? A.pe + (size_t)b * T * C : nullptr;
  auto cpos = [&](int u) { return dir == 0 ? u : Lb - u; };
  auto soff_at = [&](int u, int c) -> double {
    const int t = cpos(u);
    if (dir == 0) return (ps_b && t < T) ? (double)ps_b[(size_t)t * C + c] : 0.0;
    return (pe_b && t >= 1) ? (double)pe_b[(size_t)(t - 1) * C + c] : 0.0;
  };
  auto toff_at = [&](int u, int c) -> double {
    const int t = cpos(u);
    if (dir == 0) return (pe_b && t >= 1) ? (double)pe_b[(size_t)(t - 1) * C + c] : 0.0;
    return (ps_b && t < T) ? (double)ps_b[(size_t)t * C + c] : 0.0;
  };
  auto cumd = [&](int u, int c) -> double { return (double)cum_b[(size_t)cpos(u) * C + c]; };

  // ---- constants ----------------------------------------------------------
  for (int i = tid; i < CP; i += NT) {
    dbmax[i] = i < C ? (double)L.dbmax[i] : 0.0;
    colmax[i] = i < C ? (double)A.colmax[i] : 0.0;
    edb[i] = i < C ? exp((double)L.dbmax[i]) : 0.0;
    ecm[i] = i < C ? exp((double)A.colmax[i]) : 0.0;
  }
  for (int i = tid; i < C * C; i += NT) mx[i] = A.mx[i];
  for (int i = tid; i < pl.kx * Cs; i += NT) {
    const int k = i / Cs, cc = i % Cs;
    dbd[i] = cc < C ? L.dbe[k * C + cc] : 0.0;
  }
  for (int i = tid; i < R * Cs; i += NT) ring[i] = 0.0;
  __syncthreads();

  const int c = tid;  // serial lane label
  const bool cv = serial && c < C;
  double* atab_b = A.a_tab ? A.a_tab + (size_t)b * (T + 1) * C : nullptr;
  double* Atab_b = A.A_tab ? A.A_tab + (size_t)b * (T + 1) * C : nullptr;
  double* ntab_b = A.n_tab ? A.n_tab + (size_t)b * (T + 1) : nullptr;

  // ---- initial state (position u_begin, "block -1") ----------------------
  // frame of block -1: n = 0, anchor cA_{-1} = cum(u_begin)
  double a0 = 0.0;
  if (serial) {
    double ym0;
    if (dir == 0) {
      a0 = cv ? 1.0 : 0.0;
      // ym0 = sum_c' Mx[c',c] (alpha[0] = 0 for every label)
      double y = 0.0;
      if (cv)
        for (int q = 0; q < C; ++q) y += (double)mx[q * C + c];
      ym0 = y;
    } else {
      ym0 = cv ? exp(-colmax[c]) : 0.0;  // beta[Lb] = 0
    }
    if (cv) {
      const double e0 = ym0 * exp(colmax[c] + soff_at(u_begin, c));
      ring[(R - 1) * Cs + c] = e0;  // slot of position u_begin
      const int t0 = cpos(u_begin);
      if (jc == 0 && atab_b) atab_b[(size_t)t0 * C + c] = a0;
      if (jc == 0 && Atab_b) Atab_b[(size_t)t0 * C + c] = ym0 * exp(colmax[c]);
      cA[3 * CP + c] = cumd(u_begin, c);  // anchor of block -1 (slot (-1) mod 4 = 3)
    }
    if (tid == 0) {
      if (jc == 0 && ntab_b) ntab_b[cpos(u_begin)] = 0.0;
      nring[lidx(-1)] = 0.0;
    }
  }
  __syncthreads();

  // log sources (log E + n of the block) of the kcap positions ending at ux,
  // for the chunk hand-off: [kcap][C], row r = position ux - r
  auto export_state = [&](int kind, int ux, int t0, int nt) {
    double* out = A.hand + (((size_t)b * nch + jc) * 2 + kind) * (size_t)kcap * C;
    for (int i = t0; i < kcap * C; i += nt) {
      const int s = ux - i / C, cc = i % C;
      double v = -INFINITY;
      if (s >= u_begin) {
        const int rel = s - u_begin - 1;  // -1: the start position (block -1)
        const int slot = rel >= 0 ? rel % R : R - 1;
        const double e = ring[(size_t)slot * Cs + cc];
        if (e > 0.0) v = log(e) + nring[lidx(rel >= 0 ? rel / LP : -1)];
      }
      out[i] = v;
    }
  };
  // block whose last position is u_out (the end of the warm-up)
  const int tau_out = (jc > 0 && A.hand) ? (u_out - u_begin) / LP - 1 : -10;

  WT_DECL
  if (idle) {
    // co-resident with a serial warp: stay out of its way
  } else if (!serial) {
    // =====================================================================
    // bulk warps
    // =====================================================================
    // This thread's (target, label) elements of a block for the g/h step,
    // fixed for the whole chain, and their cum values prefetched one block
    // ahead so that no global-load latency sits inside prepare().
    constexpr int kMaxE = (LP * CP + NBT - 1) / NBT;
    int e_i[kMaxE], e_c[kMaxE];
    double pre[kMaxE];
#pragma unroll
    for (int r = 0; r < kMaxE; ++r) {
      const int w = btid + r * NBT;
      e_i[r] = (w < LP * C) ? w / C : -1;
      e_c[r] = (w < LP * C) ? w % C : 0;
      pre[r] = 0.0;
    }
    // frame-table entries this thread updates: label wc, blocks q = wq0 + m*wqs
    const int QW = min(NWT, (kcap + LP - 1) / LP + 4);  // blocks a k-window reaches
    const int wc = btid % C, wq0 = btid / C, wqs = NBT / C > 0 ? NBT / C : 1;
    const bool wact = btid < wqs * C;
    // single-label far-sum item of this thread: label fc, source blocks
    // q = fqa .. fqa + BPC - 1, and their duration lags fqa*LP - (LP-1) + m
    // (m < BPC*LP + LP - 1) held in registers; lags outside 2*LP..kcap are 0
    // (the serial warp's window covers durations 1 .. 2*LP-1)
    const int fc = btid % C, fj = btid / C;
    const bool fact = BPC > 0 && fj < pl.nsplit1;
    const int fqa = 2 + fj * BPC;
    constexpr int NW = BPC > 0 ? BPC * LP + LP - 1 : 1;
    double dw[NW];
#pragma unroll
    for (int m = 0; m < NW; ++m) {
      const int k = fqa * LP - (LP - 1) + m;
      dw[m] = (BPC > 0 && fact && k >= 2 * LP && k < pl.kx) ? dbd[k * Cs + fc] : 0.0;
    }

    // The bulk work of block tau splits in two.  precompute(tau) needs only
    // the inputs: the block's anchors cA (cum at its first position), the
    // factor exp(csign*(cA_tau - cA_tau-1)) of the anchor change, and the g / h
    // factors of its targets; it runs a block ahead, after the FULL arrive of
    // the block before.  critical(tau) depends on the chain's state: the
    // normaliser n_tau = e_tau * ln 2 (an integer exponent, so a frame change
    // is an exact power of two), the frame factors W, the far sums.
    int e_m1 = 0, e_m2 = 0;  // exponents of blocks tau-1 and tau-2 (block -1: 0)
    int lend3e = 0;          // scale exponent at the end of block tau-3 (block -1: 0)
    double pre0[kMaxE];      // cum at the first position of the block, per element label
    auto prefetch_cum = [&](int tau) {
      const int u0 = u_begin + 1 + tau * LP;
#pragma unroll
      for (int r = 0; r < kMaxE; ++r) {
        const bool in = e_i[r] >= 0 && u0 + e_i[r] <= u_end;
        pre[r] = in ? cumd(u0 + e_i[r], e_c[r]) : 0.0;
        pre0[r] = (e_i[r] >= 0 && u0 <= u_end) ? cumd(u0, e_c[r]) : 0.0;
      }
    };
    auto precompute = [&](int tau) {
      const int sl = tau & 3, sp = (tau + 3) & 3;  // this block's slot, the previous block's
      const int u0 = u_begin + 1 + tau * LP;
      const int nP = (u_end - u0 + 1) < LP ? (u_end - u0 + 1) : LP;
      const bool noproj = ps_b == nullptr && pe_b == nullptr;
#pragma unroll
      for (int r = 0; r < kMaxE; ++r) {
        const int i = e_i[r], cc = e_c[r];
        if (i == 0) {
          // the thread that holds label cc's first position owns its anchor
          // in every block, so it reads the previous anchor it wrote itself
          const double da = csign * (pre[r] - cA[sp * CP + cc]);
          cA[sl * CP + cc] = pre[r];
          dar[sl * CP + cc] = da;
          dae[sl * CP + cc] = exp(fmin(fmax(da, -700.0), 700.0));
        }
        if (i >= 0 && i < nP) {
          const int u = u0 + i;
          const double d = csign * (pre[r] - pre0[r]);
          if (noproj) {
            // |dc| <= 650 keeps exp(dc) and its reciprocal normal
            if (L.ovf && fabs(d) > 650.0) *L.ovf = 1;
            const double dc = fmin(fmax(d, -650.0), 650.0);
            const double ed = exp(dc);
            gb[(sl * LP + i) * CP + cc] = edb[cc] * ed;
            hb[(sl * LP + i) * CP + cc] = ecm[cc] * __drcp_rn(ed);
          } else {
            const double gx = toff_at(u, cc) + dbmax[cc] + d, hx = colmax[cc] + soff_at(u, cc) - d;
            if (L.ovf && (gx > 700.0 || hx > 700.0)) *L.ovf = 1;
            gb[(sl * LP + i) * CP + cc] = exp(fmin(gx, 700.0));
            hb[(sl * LP + i) * CP + cc] = exp(fmin(hx, 700.0));
          }
        }
      }
      prefetch_cum(tau + 1);
    };
    // critical(tau): normaliser, frame factors and far sums of block tau
    // (far sums into buffer tau & 1); every bulk thread derives e_tau itself
    auto critical = [&](int tau) {
      const int bf = tau & 1, sl = tau & 3;
      const int u0 = u_begin + 1 + tau * LP;
      int e_tau = 0;
      if (tau >= 2) {
        const double* al = alast + ((tau - 2) & 1) * CP;
        double m;
        if (serial_scale) {
          m = SW > 1 ? fmax(al[0], al[1]) : al[0];
        } else {
          m = fmax(al[lane], CP > 32 ? al[(lane + 32) & (CP - 1)] : 0.0);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
        }
        // the block-end scale as a power of two (its binary exponent)
        const int xm = m > 0.0 ? (int)((__double_as_longlong(m) >> 52) & 0x7ff) - 1023 : 0;
        const int l2e = e_m2 + xm;
        const int gre = min(max(l2e - lend3e, -216), 216);  // 216 ln 2 = 149.7
        e_tau = l2e + 2 * gre;
        lend3e = l2e;
      }
      if (btid == 0) nring[lidx(tau)] = (double)e_tau * 0.6931471805599453;
      // frame tau-1 -> tau: w = 2^(e_tau-1 - e_tau) * exp(csign*(cA_tau - cA_tau-1)),
      // per label, computed by each thread for the label it updates
      const int de = e_m1 - e_tau;
      if (wact) {
        const double wl = ldexp(dae[sl * CP + wc], de);  // w_{tau-1}
        if (L.ovf && fabs(de * 0.6931471805599453 + dar[sl * CP + wc]) > 700.0) *L.ovf = 1;
        if (wq0 == 0) wprev[bf * CP + wc] = wl;
        double* wcur = wt + (size_t)bf * NWT * Cs;
        const double* wold = wt + (size_t)(bf ^ 1) * NWT * Cs;
        for (int q = wq0; q < QW; q += wqs) {
          double v;
          if (q == 0) {
            v = 1.0;
          } else if (tau == 0) {
            v = (q == 1) ? wl : 0.0;  // only block -1 exists
          } else {
            v = wold[(q - 1) * Cs + wc] * wl;
          }
          wcur[q * Cs + wc] = v;
        }
      }
      e_m2 = e_m1;
      e_m1 = e_tau;
      bar_sync(kBarBulk, NBT);
      WT_ADD(2);
      // far sums over sources s in [s_lo, s_hi], s_hi = u0-LP-1 (end of block tau-2).
      // Source block q (q >= 2 blocks back) holds positions sb = u0 - q*LP ..
      // sb + LP - 1 in ring slots ((tau - q) mod NR)*LP ..; for target i and
      // source r the duration is q*LP + i - r, so one block contributes an
      // LP x LP tile from a window of 2*LP-1 Db values, and block q+1's window
      // shares LP-1 of them.  An item is a label pair and a chunk of
      // consecutive source blocks; the frame factor W is one lookup per block.
      const int s_lo = (u0 - kcap) > u_begin ? (u0 - kcap) : u_begin;
      const int qmax = (u0 - s_lo + LP - 1) / LP;  // the block holding s_lo
      const int nq = qmax - 1;                      // blocks q = 2 .. qmax
      const int nsplit = BPC > 0 ? pl.nsplit1 : pl.nsplit, np = pl.np;
      const double* wcur = wt + (size_t)bf * NWT * Cs;
      if (BPC > 0 && nq > 0) {
        if (fact) {
          double acc[LP];
#pragma unroll
          for (int i = 0; i < LP; ++i) acc[i] = 0.0;
          // ring block of source block q = fqa + mq, stepped down with wrap
          // (no division per block)
          int bq = (tau - fqa) % NR;
          if (bq < 0) bq += NR;
#pragma unroll
          for (int mq = 0; mq < BPC; ++mq) {
            // every load is in bounds and unconditional (blocks past qmax and
            // sources before s_lo contribute zeros), so that the compiler can
            // issue a block's loads while the previous block's FMAs run
            const int q = fqa + mq;
            const bool qok = q <= qmax;
            const int sb = u0 - q * LP;
            const double* rp = ring + (size_t)bq * LP * Cs + fc;
            const double Wq = wcur[(q < NWT ? q : NWT - 1) * Cs + fc];
            double x[LP];
#pragma unroll
            for (int r = 0; r < LP; ++r) {
              const double v = rp[(size_t)r * Cs];
              x[r] = (qok && sb + r >= s_lo) ? v * Wq : 0.0;
            }
#pragma unroll
            for (int r = 0; r < LP; ++r)
#pragma unroll
              for (int i = 0; i < LP; ++i)
                acc[i] = fma(x[r], dw[mq * LP + (LP - 1) + i - r], acc[i]);
            bq = bq == 0 ? NR - 1 : bq - 1;
          }
#pragma unroll
          for (int i = 0; i < LP; ++i) part[(fj * LP + i) * Cs + fc] = acc[i];
        }
        bar_sync(kBarBulk, NBT);
        WT_ADD(3);
        for (int w = btid; w < LP * C; w += NBT) {
          const int i = w / C, cc = w % C;
          double s = 0.0;
          for (int j = 0; j < nsplit; ++j) s += part[(j * LP + i) * Cs + cc];
          farb[(bf * LP + i) * CP + cc] = s;
        }
      } else if (nq > 0) {
        const int bpc = (nq + nsplit - 1) / nsplit;  // source blocks per chunk
        for (int w = btid; w < np * nsplit; w += NBT) {
          const int c0 = 2 * (w % np), j = w / np;
          double acc[LP][2];
#pragma unroll
          for (int i = 0; i < LP; ++i) acc[i][0] = acc[i][1] = 0.0;
          const int qa = 2 + j * bpc, qb = min(qa + bpc - 1, qmax);
          double d[2 * LP - 1][2];
          if (qa <= qb) {
            const double2* dp = reinterpret_cast<const double2*>(dbd + (size_t)(qa * LP - (LP - 1)) * Cs + c0);
#pragma unroll
            for (int m = 0; m < 2 * LP - 1; ++m) {
              const double2 v = dp[(size_t)m * (Cs / 2)];
              // durations below 2*LP are the serial warp's window
              const bool near = qa * LP - (LP - 1) + m < 2 * LP;
              d[m][0] = near ? 0.0 : v.x;
              d[m][1] = near ? 0.0 : v.y;
            }
          }
          for (int q = qa; q <= qb; ++q) {
            const int sb = u0 - q * LP;
            int bq = (tau - q) % NR;
            if (bq < 0) bq += NR;
            const double2* rp = reinterpret_cast<const double2*>(ring + (size_t)bq * LP * Cs + c0);
            const double2 Wq = *reinterpret_cast<const double2*>(wcur + q * Cs + c0);
            double x[LP][2];
#pragma unroll
            for (int r = 0; r < LP; ++r) {
              const double2 e = rp[(size_t)r * (Cs / 2)];
              const bool ok = sb + r >= s_lo;
              x[r][0] = ok ? e.x * Wq.x : 0.0;
              x[r][1] = ok ? e.y * Wq.y : 0.0;
            }
#pragma unroll
            for (int r = 0; r < LP; ++r)
#pragma unroll
              for (int i = 0; i < LP; ++i) {
                acc[i][0] = fma(x[r][0], d[LP - 1 + i - r][0], acc[i][0]);
                acc[i][1] = fma(x[r][1], d[LP - 1 + i - r][1], acc[i][1]);
              }
            if (q < qb) {
#pragma unroll
              for (int m = 0; m < LP - 1; ++m) {
                d[m][0] = d[m + LP][0];
                d[m][1] = d[m + LP][1];
              }
              const double2* dn = reinterpret_cast<const double2*>(dbd + (size_t)((q + 1) * LP) * Cs + c0);
#pragma unroll
              for (int m = LP - 1; m < 2 * LP - 1; ++m) {
                const double2 v = dn[(size_t)(m - (LP - 1)) * (Cs / 2)];
                d[m][0] = v.x;
                d[m][1] = v.y;
              }
            }
          }
#pragma unroll
          for (int i = 0; i < LP; ++i) {
            part[(j * LP + i) * Cs + c0] = acc[i][0];
            part[(j * LP + i) * Cs + c0 + 1] = acc[i][1];
          }
        }
        bar_sync(kBarBulk, NBT);
        WT_ADD(3);
        for (int w = btid; w < LP * C; w += NBT) {
          const int i = w / C, cc = w % C;
          double s = 0.0;
          for (int j = 0; j < nsplit; ++j) s += part[(j * LP + i) * Cs + cc];
          farb[(bf * LP + i) * CP + cc] = s;
        }
      } else {
        for (int w = btid; w < LP * C; w += NBT) {
          const int i = w / C, cc = w % C;
          farb[(bf * LP + i) * CP + cc] = 0.0;
        }
      }
      // (bar.arrive orders these shared-memory writes before the serial
      // warp's bar.sync on FULL: no separate fence)
      WT_ADD(4);
    };

    prefetch_cum(0);
    if (NB > 0) {
      precompute(0);
      critical(0);
      bar_arrive(kBarFull0, NPART);
    }
    if (NB > 1) {
      precompute(1);
      critical(1);
      bar_arrive(kBarFull1, NPART);
    }
    if (NB > 2) precompute(2);
    for (int tau = 2; tau < NB + 2; ++tau) {
      WT_ADD(5);
      // buffer (tau & 1) is free once the serial warp is done with block tau-2
      bar_sync(((tau - 2) & 1) ? kBarDone1 : kBarDone0, NPART);
      WT_ADD(0);

      // the warm-up is over: hand off this chunk's guess of the state
      if (tau - 2 == tau_out) export_state(0, u_out, btid, NBT);
      if (tau < NB) {
        critical(tau);
        bar_arrive((tau & 1) ? kBarFull1 : kBarFull0, NPART);
      }
      {
        // block tau-2 is final: its normalisers to global memory, past the
        // warm-up only (the serial warp writes the a and A rows itself)
        const int tb = tau - 2;
        const int ub0 = u_begin + 1 + tb * LP;
        const int nPb = (u_end - ub0 + 1) < LP ? (u_end - ub0 + 1) : LP;
        if (btid < nPb && ub0 + btid > u_out && ntab_b) ntab_b[cpos(ub0 + btid)] = nring[lidx(tb)];
      }
      // the next block's input-only factors (its slot (tau+1) mod 4 was last
      // read by the serial warp in block tau-3, which is done)
      if (tau + 1 < NB) precompute(tau + 1);
    }
    WT_FLUSH(0);
  } else {
    // =====================================================================
    // serial warp(s)
    // =====================================================================
    const double ecol = cv ? exp(colmax[c]) : 0.0;
    double dbk[2 * LP];  // Db[k] for k = 0 .. 2LP-1 (index 0 unused)
#pragma unroll
    for (int k = 0; k < 2 * LP; ++k) dbk[k] = (cv && k >= 1) ? dbd[k * Cs + c] : 0.0;
    auto sync_serial = [&]() {
      if (SW == 1)
        __syncwarp();
      else
        bar_sync(kBarSerial, CP);
    };
    auto group_sumd = [&](double v) -> double {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (SW == 1) return v;
      if (lane == 0) misc[8 + warp] = v;
      bar_sync(kBarSerial, CP);
      double r = misc[8] + misc[9];
      bar_sync(kBarSerial, CP);
      return r;
    };

    double a_last = a0;
    double n_last = 0.0;
    // The block loop, instantiated for MV mat-vec terms (C rounded up to a
    // multiple of 8 when one warp holds the labels, CP otherwise), so that a
    // chain of C = 24 labels issues 24 float64 FMAs per position, not 32.
    auto run_serial = [&](auto mv_tag) {
      constexpr int MV = decltype(mv_tag)::value;
      double mxr[CP == 32 ? MV : 1];
#pragma unroll
      for (int q = 0; q < (CP == 32 ? MV : 1); ++q)
        mxr[q] = (CP == 32 && cv && q < C) ? mx[q * C + c] : 0.0;
      // the mat-vec in two halves: publish this lane's a into the exchange
      // buffer of parity par, then (after independent work) read the whole
      // vector and form ym.  The buffers alternate by position, so no
      // barrier is needed after the reads: a lane writes buffer par again
      // only two positions later, past the next position's barrier, which
      // every lane reaches after its reads of this one.
      auto mv_publish = [&](double a, int par) { abuf[par * CP + c] = cv ? a : 0.0; };
      auto mv_finish = [&](int par) -> double {
        const double* ab = abuf + par * CP;
        sync_serial();
        double y[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) y[q] = 0.0;
        if (CP == 32) {
          const double2* ab2 = reinterpret_cast<const double2*>(ab);
#pragma unroll
          for (int q = 0; q < MV / 2; ++q) {
            const double2 v = ab2[q];
            y[(2 * q) & 7] = fma(v.x, mxr[2 * q], y[(2 * q) & 7]);
            y[(2 * q + 1) & 7] = fma(v.y, mxr[2 * q + 1], y[(2 * q + 1) & 7]);
          }
        } else if (cv) {
          const double2* ab2 = reinterpret_cast<const double2*>(ab);
#pragma unroll 4
          for (int q = 0; q < CP / 2; ++q) {
            const double2 v = ab2[q];
            const int q0 = 2 * q, q1 = 2 * q + 1;
            y[q0 & 7] = fma(v.x, q0 < C ? mx[q0 * C + c] : 0.0, y[q0 & 7]);
            y[q1 & 7] = fma(v.y, q1 < C ? mx[q1 * C + c] : 0.0, y[q1 & 7]);
          }
        }
        return ((y[0] + y[1]) + (y[2] + y[3])) + ((y[4] + y[5]) + (y[6] + y[7]));
      };

      // near window: win[j] = E[u-1-j] for the next target u, j < NWIN, in the
      // current block's frame (the far sums cover durations NWIN+1 and up)
      constexpr int NWIN = 2 * LP - 1;
      double win[NWIN];
#pragma unroll
      for (int j = 0; j < NWIN; ++j) win[j] = 0.0;
      win[0] = cv ? ring[(R - 1) * Cs + c] : 0.0;  // position u_begin
      int mpar = 0;
      for (int tau = 0; tau < NB; ++tau) {
        const int bf = tau & 1, sl = tau & 3;
        WT_ADD(12);
        bar_sync(bf ? kBarFull1 : kBarFull0, NPART);
        WT_ADD(8);
        const int u0 = u_begin + 1 + tau * LP;
        const int nP = (u_end - u0 + 1) < LP ? (u_end - u0 + 1) : LP;
        const double n_tau = nring[lidx(tau)];
        // the window's sources are in the previous blocks' frames: one factor
        // w_{tau-1} brings all of them to this block's
        const double wp = cv ? wprev[bf * CP + c] : 0.0;
        const double* far_b = farb + (size_t)bf * LP * CP + c;
        const double* g_b = gb + (size_t)sl * LP * CP + c;
        const double* h_b = hb + (size_t)sl * LP * CP + c;
        // the factors of the first two positions; each position then loads
        // the ones two positions ahead, so that no shared-memory load (which
        // queues behind the bulk warps' traffic) sits on the critical path
        double gA = g_b[0], hA = h_b[0];
        double gB = g_b[CP], hB = h_b[CP], fB = far_b[CP];
#pragma unroll
        for (int j = 0; j < NWIN; ++j) win[j] *= wp;
        // R = far sum + the window's terms of durations 2 .. NWIN+1 ... of the
        // first target; the newest source's term (duration 1) is added when it
        // is known
        double rn;
        {
          double q4[4] = {cv ? far_b[0] : 0.0, 0.0, 0.0, 0.0};
#pragma unroll
          for (int j = 0; j + 1 < NWIN; ++j) q4[j & 3] = fma(win[j + 1], dbk[j + 2], q4[j & 3]);
          rn = (q4[0] + q4[1]) + (q4[2] + q4[3]);
        }
        int slot = (tau % NR) * LP;  // slot of position u0: (u0 - 1) mod R
        // one position per iteration, identical code for every position (a
        // short loop body: a block-long unrolled sequence runs slower)
#pragma unroll 1
        for (int i = 0; i < nP; ++i) {
          const double gi = gA, hcur = hA, fn = fB;
          gA = gB;
          hA = hB;
          {
            const int ip = i + 2 < LP ? i + 2 : LP - 1;  // in the block's buffers
            gB = g_b[ip * CP];
            hB = h_b[ip * CP];
            fB = far_b[ip * CP];
          }
          WT_ADD(13);
          double a = 0.0;
          if (cv) {
            const double S = fma(win[0], dbk[1], rn);
            a = (S > 0.0) ? gi * S : 0.0;
          }
          mv_publish(a, mpar);
          WT_ADD(9);
          // the next target's R from the sources known now (its duration-1
          // source is this position's, still to come), while the published
          // values become visible
          if (i + 1 < nP) {
            double q4[4] = {cv ? fn : 0.0, 0.0, 0.0, 0.0};
#pragma unroll
            for (int j = 0; j + 1 < NWIN; ++j) q4[j & 3] = fma(win[j], dbk[j + 2], q4[j & 3]);
            rn = (q4[0] + q4[1]) + (q4[2] + q4[3]);
          }
          const double ym = mv_finish(mpar);
          mpar ^= 1;
          WT_ADD(10);
          double e = 0.0;
          if (cv) {
            e = (ym > 0.0) ? ym * hcur : 0.0;
            ring[(slot + i) * Cs + c] = e;
            // table rows straight to global memory (the load/store queue,
            // not the shared-memory pipe the bulk warps keep busy)
            if (u0 + i > u_out) {
              const size_t row = (size_t)cpos(u0 + i) * C + c;
              if (atab_b) atab_b[row] = a;
              if (Atab_b) Atab_b[row] = ym * ecol;
            }
          }
#pragma unroll
          for (int j = NWIN - 1; j > 0; --j) win[j] = win[j - 1];
          win[0] = e;
          a_last = a;
          WT_ADD(11);
        }
        // the state at the end of the block, from which the bulk derives the
        // block's scale for its normaliser prediction: its per-warp maxima when
        // the bulk is the busier side (long duration windows), else the state
        if (serial_scale) {
          double mm = cv ? a_last : 0.0;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) mm = fmax(mm, __shfl_xor_sync(0xffffffffu, mm, o));
          if (lane == 0) alast[bf * CP + warp] = mm;
        } else {
          alast[bf * CP + c] = cv ? a_last : 0.0;
        }
        n_last = n_tau;
        // bar.arrive orders this block's ring and alast writes before the
        // bulk warps' bar.sync on DONE (no fence: it would also wait for the
        // table rows' global stores)
        bar_arrive(bf ? kBarDone1 : kBarDone0, NPART);
      }
    };
    if (CP == 32 && C <= 8)
      run_serial(std::integral_constant<int, 8>{});
    else if (CP == 32 && C <= 16)
      run_serial(std::integral_constant<int, 16>{});
    else if (CP == 32 && C <= 24)
      run_serial(std::integral_constant<int, 24>{});
    else
      run_serial(std::integral_constant<int, 32>{});
    WT_FLUSH(8);
    // forward output: logZ = n(Lb) + log sum_c a[Lb,c] (the chunk that ends
    // the sequence; a later chunk fix-up adds the chunk's offset)
    if (dir == 0 && u_end == Lb) {
      const double s = group_sumd(cv ? a_last : 0.0);
      if (tid == 0) {
        const double lz = (Lb == 0 || !(s > 0.0)) ? (double)kRefNegInf : n_last + log(s);
        if (A.partition) A.partition[b] = (float)lz;
        if (A.logz) A.logz[b] = lz;
      }
    }
  }
  // hand off the state at the end of a chunk that does not end the sequence
  if (A.hand && u_end < Lb) {
    __syncthreads();
    export_state(1, u_end, tid, NT);
  }
}

// ---------------------------------------------------------------------------
template <int CP, int BPC>
static cudaError_t launch_ws_cp(const LChainLaunch& L, int grid, size_t smem, cudaStream_t s) {
  auto kern = lchain_ws_kernel<CP, 8, BPC>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kWsThreads, smem, s>>>(L);
  return cudaGetLastError();
}

#ifdef SEMICRF_TIMING
extern "C" int semicrf_debug_wstiming(unsigned long long* out) {
  return (int)cudaMemcpyFromSymbol(out, g_wstim, sizeof(g_wstim));
}
#endif

cudaError_t launch_lchain_ws(const LChainLaunch& L, int grid, cudaStream_t s) {
  if (L.B <= 0 || grid <= 0) return cudaSuccess;
  WsPlan p;
  if (!ws_choose(p, L.C, L.K)) return cudaErrorInvalidValue;
  // the smallest register window that covers the plan's source blocks per
  // split; longer windows take the label-pair items
  const int need = p.bpc1;
  if (ws_cp(L.C) == 32) {
    if (need <= 1) return launch_ws_cp<32, 1>(L, grid, (size_t)p.bytes, s);
    if (need <= 2) return launch_ws_cp<32, 2>(L, grid, (size_t)p.bytes, s);
    if (need <= 3) return launch_ws_cp<32, 3>(L, grid, (size_t)p.bytes, s);
    if (need <= 5) return launch_ws_cp<32, 5>(L, grid, (size_t)p.bytes, s);
    if (need <= 7) return launch_ws_cp<32, 7>(L, grid, (size_t)p.bytes, s);
    return launch_ws_cp<32, 0>(L, grid, (size_t)p.bytes, s);
  }
  if (need <= 3) return launch_ws_cp<64, 3>(L, grid, (size_t)p.bytes, s);
  if (need <= 7) return launch_ws_cp<64, 7>(L, grid, (size_t)p.bytes, s);
  return launch_ws_cp<64, 0>(L, grid, (size_t)p.bytes, s);
}

}  // namespace semicrf
