// Internal declarations shared by the CUDA translation units of libsemicrf.
//
// Numerical conventions (all kernels):
//  * Scores are natural-log float32.  Every chain keeps its values relative
//    to an integer-valued per-block normaliser N (float64), so stored
//    quantities stay O(10) and differences N(s) - N(u) are exact in float32.
//  * Prefix-sum differences cum[u] - cum[s] are always formed first (they
//    are exact or nearly so) before small terms are added.
//  * "-inf" is a real IEEE -inf internally; the reference's NEG_INF (-1e9)
//    only appears at the API boundary (checkpoints of unreached positions,
//    the partition of an empty sequence).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/semicrf.h"

namespace semicrf {

constexpr float kNegInf = -__builtin_huge_valf();
constexpr float kRefNegInf = -1e9f;  // streaming/constants.py:10

// ---------------------------------------------------------------------------
// small device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ex(float x) {  // e^x, x <= 0 in all uses that matter
  return __expf(x);
}
__device__ __forceinline__ float lg(float x) { return __logf(x); }

__device__ __forceinline__ float warp_max(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------
// per-launch constants prepared by prep_kernel (chain.cu)
// ---------------------------------------------------------------------------
struct Prepared {
  // mat-vec operand for the forward chain (M = transition) and the backward
  // chain (M = transition^T): max semiring M (float32); log semiring
  // exp(M - colmax) in float64 (mxd_*), together with dbed = exp(dbl - dbmax)
  float* mx_f;
  float* mx_b;
  double* mxd_f;
  double* mxd_b;
  double* dbed;     // (KX, C), log semiring
  float* colmax_f;  // (C)
  float* colmax_b;
  float* dbl;       // (KX, C): log duration bias by duration k, -inf outside 1..kcap
  float* dbe;       // (KX, C): exp(dbl - dbmax)
  float* dbmax;     // (C)
  int* ovf;         // log semiring: the chain's overflow flag
  int kx;           // rows of dbl / dbe = kcap + P + 1
};

// One chain role (see chain.cu for the algorithm).
struct ChainArgs {
  int mode;   // 0 = whole sequence, 1 = one checkpoint segment (restart)
  int dir;    // 0 = forward (alpha), 1 = backward (beta)
  // inputs
  const float* cum;
  const float* ps;
  const float* pe;
  const int64_t* lengths;
  // prepared constants
  const float* mx;
  const float* colmax;
  // forward outputs
  float* partition;      // (B)
  double* logz;          // (B)
  float* ref_ckpt;       // (B, nref, K, C) reference layout, or null
  int nref;
  int sref;
  // restart state
  float* sv_f;           // (B, nint, kcap*C + 2*C)
  double* sv_d;          // (B, nint, kcap)
  int nint;
  int sint;              // multiple of P
  int write_saved;
  // tables indexed by cum position t, or null
  float* tab_x;          // (B, T+1, C)
  float* tab_m;          // (B, T+1, C)
  double* tab_n;         // (B, T+1)
  // Viterbi
  int16_t* bp_k;         // (B, T+1, C)
  uint8_t* bp_c;         // (B, T+1, C)
  int* final_c;          // (B)
  float* score;          // (B) max-semiring score
};

struct ChainLaunch {
  int B, T, K, C, kcap;
  Prepared prep;
  int n1;          // CTAs [0, n1) run role a0, [n1, grid) run role a1
  ChainArgs a0;
  ChainArgs a1;
};

// float64 linear-domain log-semiring chain (lchain.cu)
struct LChainArgs {
  int mode;  // 0 = whole sequence, 1 = checkpoint segment (forward only)
  int dir;   // 0 = forward (alpha), 1 = backward (beta)
  const float* cum;
  const float* ps;
  const float* pe;
  const int64_t* lengths;
  const double* mx;      // exp(M - colmax), float64 (C*C)
  const float* colmax;   // (C)
  // forward outputs
  float* partition;
  double* logz;
  float* ref_ckpt;
  int nref;
  int sref;
  // restart states (checkpoint mode)
  double* sv;
  int nint;
  int sint;
  int write_saved;
  // chain tables, indexed by cum position t: a = exp(x - n), A = exp(m - n)
  // and the normaliser n per position (x = alpha, m = A for dir 0; x = G,
  // m = beta for dir 1)
  double* a_tab;
  double* A_tab;
  double* n_tab;
  // time chunks (lchain_ws only): the chain of a sequence is split into
  // nchunk chunks of chunk_len positions (u); chunk j > 0 starts warm
  // positions early from a uniform state and writes outputs only past
  // j*chunk_len.  hand receives, per (sequence, chunk), the log sources of the
  // last kcap positions at j*chunk_len (kind 0) and at the chunk's end (kind
  // 1): [B][nchunk][2][kcap][C].
  int nchunk;
  int chunk_len;
  int warm;
  double* hand;
  const int* only;  // if set, only sequences b with only[b] != 0 run
};
struct LChainLaunch {
  int B, T, K, C;
  const double* dbe;   // (kx, C) exp(db - dbmax), zero outside durations 1..kcap
  const float* dbmax;  // (C)
  const float* dbl;    // (kx, C) log duration bias by duration (the log-domain fallback)
  int* ovf;            // set by lchain_ws_kernel when an exponent clamp clips; may be null
  int n1;              // CTAs [0, n1) run a0, the rest a1
  LChainArgs a0;
  LChainArgs a1;
};
// Number of SMs of the current device (cudaDevAttrMultiProcessorCount),
// cached per device index; launch planning sizes grids and time chunks by it.
int device_sm_count();
cudaError_t launch_lchain(const LChainLaunch& L, int grid, cudaStream_t s);
// warp-specialised variant for C <= 64, whole-sequence chains (mode 0) only
cudaError_t launch_lchain_ws(const LChainLaunch& L, int grid, cudaStream_t s);
// lchain_fix.cu: log-domain rerun of the lchain_ws chains when L.ovf is set
bool lchain_fix_supported(int C, int K);
cudaError_t launch_lchain_fix(const LChainLaunch& L, int grid, cudaStream_t s);
// cluster variant for 64 < C <= 256 (lchain_cl.cu): one chain per cluster of
// four CTAs, whole-sequence chains (mode 0) without ring checkpoints
bool lchain_cl_supported(int C, int K);
cudaError_t launch_lchain_cl(const LChainLaunch& L, int nchains, cudaStream_t s);

// time chunking of the float64 chains (lchunk.cu)
struct ChunkPlan {
  int nchunk, len, warm;
  int warm2;  // > 0: sequences whose chunks do not join rerun their chunks with this warm-up
};
// chunks for B sequences (times nroles chains each) of length T; nchunk = 1
// means no chunking.  warm_override > 0 forces chunking with that warm-up.
ChunkPlan chunk_plan(int B, int T, int K, int C, int nroles, int warm_override);
size_t chunk_hand_doubles(int B, int K, int C, const ChunkPlan& cp);
// compares the boundary states, accumulates the per-chunk log offsets D, and
// adds them to the tables (n_tab) and log Z; sequences whose states do not
// agree get fail[b] = 1 and are left for a serial rerun
struct ChunkFix {
  int B, T, K, C, dir;
  ChunkPlan cp;
  const int64_t* lengths;
  const double* hand;
  double* rdiff;  // [B][nchunk]
  int* okf;       // [B][nchunk]
  double* D;      // [B][nchunk]
  int* fail;      // [B]
  const int* only;  // null, or [B]: check and fix only the sequences flagged here
  double* n_tab;  // (B, T+1) or null
  double* logz;   // (B) or null
  float* partition;
};
// both chains (f0: alpha, f1: beta) in one launch per step
cudaError_t launch_chunk_fix(const ChunkFix& f0, const ChunkFix& f1, cudaStream_t s);
bool lchain_ws_supported(int C, int K);
bool lchain_supported(int C, int K);
size_t lchain_saved_doubles(int C, int K);       // restart record per checkpoint
constexpr int kPrepRowsExtra = 17;  // dbl/dbe rows = kcap + kPrepRowsExtra

// log-semiring gradients from the alpha and beta chain tables (lmarg.cu)
struct LMargArgs {
  int B, T, K, C, kcap;
  const float* cum;
  const float* ps;
  const float* pe;
  const float* tr;  // (C, C)
  const float* db;  // (K, C)
  const int64_t* lengths;
  const double* logz;
  const float* grad_output;
  const double* xa;  // alpha chain: exp(alpha - xn), exp(A - xn), xn
  const double* xA;
  const double* xn;
  const double* ya;  // beta chain: exp(G - yn), exp(beta - yn), yn
  const double* yA;
  const double* yn;
  float* grad_cum;
  float* grad_ps;
  float* grad_pe;
  double* la;       // (B, T+1, C) block-relative linear start factors exp(log la - maX)
  double* lb;       // (B, T+1, C) block-relative linear end factors exp(log lb - mbY)
  double* maX;      // (B, nblk, C) block references of log la: within ln 2 above the maximum
  double* mbY;      // (B, nblk, C) block references of log lb: within ln 2 above the maximum
  double* part_tr;  // (B, nchunk, C*C)
  int nchunk;
  double* part_db;  // (B, nsplit, kcap, C)
  int nsplit;
  int cg;           // labels per duration CTA
  int* dbflag;      // (B) set when a duration tile's block factor nears the float64 range
};
struct LMargPlan {
  int nchunk, nsplit, cg, ncg, mi, nblk;
  size_t db_smem;
  bool ok;
};
LMargPlan lmarg_plan(int B, int T, int K, int C);
cudaError_t launch_lmarg(const LMargArgs& a, float* grad_tr, float* grad_db, cudaStream_t s);

// launchers (chain.cu)
cudaError_t launch_prep(const float* tr, const float* db, int K, int C, int kcap, int P,
                        int semiring, const Prepared& prep, cudaStream_t s);
cudaError_t launch_chain(const ChainLaunch& L, int grid, int semiring, bool backpointers,
                         cudaStream_t s);
int chain_block_size(int C);  // P used by launch_chain for this C
size_t chain_smem_bytes(int C, int K, int semiring, bool backpointers);
bool chain_supported(int C, int K, int semiring, bool backpointers);

// marginals.cu
struct MargArgs {
  int B, T, K, C, kcap;
  const float* cum;
  const float* ps;
  const float* pe;
  const float* tr;
  const float* dbl;
  const int64_t* lengths;
  const double* logz;
  const float* grad_output;
  const float* xa; const float* ma; const double* na;
  const float* xb; const float* mb; const double* nb;
  float* grad_cum;
  float* grad_ps;
  float* grad_pe;
  float* part_tr;  // (B, C*C) per-sequence transition gradients
  float* part_db;  // (B, K*C) per-sequence duration-bias gradients
};
// semiring 0 = log, 1 = max; alse / pstart are (B, T+1, C) scratch tables
cudaError_t launch_marginals_impl(const MargArgs& a, int semiring, float* alse, float* pstart,
                                  cudaStream_t s);
cudaError_t launch_reduce_shared(const MargArgs& a, float* grad_tr, float* grad_db,
                                 cudaStream_t s);

// vchain.cu: max-semiring chain for C <= 32, one warp per sequence
struct VChainArgs {
  int B, T, K, C;
  const float* cum;
  const float* tr;
  const float* db;
  const float* ps;
  const float* pe;
  const int64_t* lengths;
  float* partition;  // (B) score, may be null
  double* logz;      // (B) score in float64, may be null
  int* final_c;      // (B) first maximising final label, may be null
  int16_t* bp_k;     // (B, T+1, C) winning duration, may be null
  uint8_t* bp_c;     // (B, T+1, C) winning source label, may be null
  uint16_t* bp;      // (B, T+1, C) packed: duration | (source label at the start) << 8
};
bool vchain_supported(int B, int C, int K);
cudaError_t launch_vchain(const VChainArgs& a, cudaStream_t s);

// kcc.cu -- duration-dependent transitions, transition of shape (K, C, C)
struct KccPrep {
  double* ef;   // (K, C, C) exp(tr[k][c',c] - tf[k][c])        (forward chain, marginals)
  double* eb;   // (K, C, C) [k][c2][c] = exp(tr[k][c,c2] - tb[k][c])   (beta chain)
  double* tf;   // (K, C) max over c' of tr[k][c',c]
  double* tb;   // (K, C) max over c2 of tr[k][c,c2]
  double* tdf;  // (K, C) tf + db
  double* rf;   // max semiring: (K, C, C) [k][c'][c] = tr[k][c',c] + db[k,c]
  double* rb;   // max semiring: (K, C, C) [k][c2][c] = tr[k][c,c2] + db[k,c2]
  // log semiring, blocked chain (kblk.cu): fk[c] = max_{k>=1,c'} tr[k][c',c] + db[k,c],
  // xf[k][m][l] = exp(tr[k][m][l] + db[k,l] - fk[l]), xb[k][m][l] = exp(tr[k][l][m] + db[k,m] - fk[m])
  double* xf;
  double* xb;
  double* fk;
};
struct KccArgs {
  int B, T, K, C, kcap, semiring;
  const float* cum;
  const float* tr;
  const float* db;
  const float* ps;
  const float* pe;
  const int64_t* lengths;
  KccPrep pr;
  // chain outputs: log tables (B, T+1, C), row maxima of alpha (B, T+1)
  double* alpha;
  double* amax;
  double* beta;
  double* logz;
  float* partition;
  float* ref_ckpt;
  int nref, sref;
  // backward
  const float* grad_output;
  float* grad_cum;
  float* grad_ps;
  float* grad_pe;
  double* st;       // (B, T+1, C) start terms of the marginals
  double* et;       // (B, T+1, C) end terms of the marginals
  double* pend;     // max semiring: end marginals (B, T+1, C)
  double* part_tr;  // (nslice, C, kcap*C) partial sums of the transition marginals
  int nslice;
  // log semiring with the blocked kernels (kblk.cu): source factors al (B, T+1, C)
  // and per-block anchors anc (B, T/16+1, C); st / et then hold the linear start
  // and end factors
  double* al;
  double* anc;
  double* ep1;  // end factors relative to the previous block's anchor
  int* kflag;    // set by the blocked factor pass when an end factor nears the float64 range
  int* gate;     // fallback pass: the per-item kernels return at once unless *gate != 0
};
bool kcc_supported(int C, int K);
size_t kcc_prep_doubles(int K, int C, int semiring);
KccPrep kcc_prep_carve(double* base, int K, int C, int semiring);
int kcc_tr_slices(int B, int K, int C);
cudaError_t launch_kcc_prep(const float* tr, const float* db, int K, int C, const KccPrep& pr,
                            cudaStream_t s);
cudaError_t launch_kcc_chains(const KccArgs& a, int ndir, cudaStream_t s);
cudaError_t launch_kcc_grads(const KccArgs& a, float* grad_tr, float* grad_db, cudaStream_t s);
// kblk.cu -- the blocked (K, C, C) chain of the log semiring
bool kblk_supported(int C, int K);
cudaError_t launch_kblk_prep(const float* tr, const float* db, int K, int C, const KccPrep& pr,
                             cudaStream_t s);
cudaError_t launch_kblk_chains(const KccArgs& a, int ndir, cudaStream_t s);
int kblk_tr_slices(int B, int K, int C);
size_t kblk_anchor_rows(int T);  // anchors per sequence and label
cudaError_t launch_kblk_grads(const KccArgs& a, cudaStream_t s);

// escan.cu -- the edge-tensor scan
bool escan_supported(int K, int C);
cudaError_t launch_escan_forward(int B, int N, int K, int C, const float* edge,
                                 const int64_t* lengths, int semiring, float* partition,
                                 double* logz, double* beta_tab, int32_t* bp, cudaStream_t s);
cudaError_t launch_escan_backward(int B, int N, int K, int C, const float* edge,
                                  const int64_t* lengths, int semiring, const double* beta,
                                  const double* logz, const int32_t* bp, const float* grad_output,
                                  float* grad_edge, double* gamma, cudaStream_t s);

// viterbi.cu
// backtrace over the packed backpointers of vchain.cu
size_t backtrace_packed_smem(int T, int C);
cudaError_t launch_backtrace_packed(int B, int T, int K, int C, const float* cum,
                                    const float* tr, const float* db, const int64_t* lengths,
                                    int64_t max_len, const uint16_t* bp, const int* final_c,
                                    int32_t* seg_start, int32_t* seg_end, int32_t* seg_label,
                                    double* seg_score, int32_t* nseg, cudaStream_t s);
cudaError_t launch_backtrace(int B, int T, int K, int C, const float* cum, const float* tr,
                             const float* db, const int64_t* lengths, int64_t max_len,
                             const int16_t* bp_k, const uint8_t* bp_c, const int* final_c,
                             int32_t* seg_start, int32_t* seg_end, int32_t* seg_label,
                             double* seg_score, int32_t* nseg, cudaStream_t s);

// gold.cu
cudaError_t launch_gold(int B, int T, int K, int C, const float* cum, const int64_t* labels,
                        const int64_t* lengths, const float* tr, const float* db, float* out,
                        cudaStream_t s);
cudaError_t launch_gold_backward(int B, int T, int K, int C, const int64_t* labels,
                                 const int64_t* lengths, const float* grad_out,
                                 float* grad_cum, float* grad_tr, float* grad_db,
                                 float* part, cudaStream_t s);

}  // namespace semicrf
