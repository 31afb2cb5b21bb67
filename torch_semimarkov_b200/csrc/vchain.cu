// vchain.cu -- max-semiring chain for C <= 32: one warp per sequence.
//
// Reference semantics: the max branch of streaming/pytorch_reference.py:
// 116-273 (forward) with the Viterbi backpointers of nn.py:444-505.  The
// factorised recurrence (exact in the max semiring):
//     x[t,c]  = pe[t-1,c] + max_{k=1..min(K',t)} ( (cum[t,c] - cum[t-k,c]) + sv[t-k,c] + db[min(k,K-1),c] )
//     m[s,c]  = max_c' ( x[s,c'] + tr[c',c] ),      sv[s,c] = m[s,c] + ps[s,c]
// with x[0,c] = 0, K' = max(1, K-1), ties to the smallest k (strict >,
// nn.py:494) and to the first c' (nn.py:491); the score is max_c x[L,c] with
// the first maximising label (nn.py:501).
//
// Float64 arithmetic on the float32 inputs.  A path score grows about
// linearly with t (to thousands at T = 2048), where float32 rounding would
// reach 1e-4 per step and flip decisions between paths whose scores differ by
// that little; in float64 only ties closer than about 1e-12 can resolve
// differently from an exact evaluation.  Each ring entry is the single double
// E[s,c] = sv[s,c] - cum[s,c], so a candidate is E[t-k,c] + db[k,c] and the
// common cum[t,c] is added to the winner only.
//
// Lane c of the warp owns label c; for C <= 16 lanes c and c + 16 both do,
// and each takes half of every maximum (durations 1..KM/2 and KM/2+1..KM,
// source labels 0..NC/2-1 and NC/2..NC-1), the halves joined by one
// shuffle that keeps the lower half on ties, so a position costs each lane
// half the candidates.  The ring of the last K' positions lives in per-warp
// shared memory that only the lanes of that label read (and the lower lane
// writes), so the recurrence needs no barrier.  A duration maximum is a tree
// over groups of up to 16 candidates (all loaded and added independently,
// then compare-select levels that keep the smaller k on ties), the groups
// combined in order; the label maximum m is shuffles and the same stable
// tree.  Several sequences run per CTA, one per warp, so a batch of B
// sequences is B warps across the GPU.

#include "semicrf_internal.cuh"

namespace semicrf {

namespace {

constexpr int kVMaxWarps = 4;
constexpr size_t kVSmemMax = 200 * 1024;
constexpr double kDNegInf = -__builtin_huge_val();

struct VPlan {
  int kcap, R, wpb;
  size_t smem;
};

inline bool vplan(VPlan& p, int B, int C, int K) {
  if (C > 32 || C < 1) return false;
  p.kcap = K > 1 ? K - 1 : 1;
  // longer duration windows: the block-parallel chain (chain.cu) spreads the
  // k-scan over a CTA and is faster than one warp's serial scan
  if (p.kcap > 64) return false;
  p.R = 1;
  while (p.R < p.kcap + 1) p.R <<= 1;
  const size_t shared = 8 * (size_t)(p.kcap + 1) * C;  // duration bias table (doubles)
  const size_t per_warp = 17 * (size_t)p.R * C;        // E ring (twice, doubles) + argmax ring
  // spread small batches over the SMs: about one warp per SM sub-partition
  const int nsm = device_sm_count();
  int wpb = (B + nsm - 1) / nsm;
  if (wpb < 1) wpb = 1;
  if (wpb > kVMaxWarps) wpb = kVMaxWarps;
  while (wpb > 1 && shared + wpb * per_warp > kVSmemMax) --wpb;
  if (shared + wpb * per_warp > kVSmemMax) return false;
  p.wpb = wpb;
  p.smem = shared + wpb * per_warp;
  return true;
}

// stable maximum of v[0..N) (N a power of two): the lowest index among equal
// maxima, as a strict > scan in index order would pick
template <int N>
__device__ __forceinline__ void stable_max(double (&v)[N], int (&ix)[N]) {
#pragma unroll
  for (int w = 1; w < N; w <<= 1)
#pragma unroll
    for (int q = 0; q < N; q += 2 * w)
      if (v[q + w] > v[q]) {  // strict: ties keep the lower index
        v[q] = v[q + w];
        ix[q] = ix[q + w];
      }
}

// NC: labels rounded up to 8/16/32 (the lanes that take part in the label
// maximum).  KM: durations rounded up to 16/32/64; the k-scan runs in groups
// of 16, with the duration-bias row held in registers up to KM = 32.
template <int NC, int KM>
__global__ void __launch_bounds__(32 * kVMaxWarps) vchain_kernel(const VChainArgs a, int kcap,
                                                                 int R, int wpb) {
  extern __shared__ __align__(16) double vsm[];
  constexpr bool HALF = NC <= 16;      // two lanes per label, each half the candidates
  constexpr int KH = HALF ? KM / 2 : KM;  // durations per lane
  constexpr int NQ = HALF ? NC / 2 : NC;  // source labels per lane
  constexpr int KG = KH < 16 ? KH : 16;   // candidates per tree
  constexpr int NG = KH / KG;             // groups
  constexpr bool kDbReg = KM <= 32;       // duration biases in registers
  const int C = a.C, K = a.K, T = a.T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  double* dbl = vsm;  // [kcap + 1][C], row k = db[min(k, K-1)]
  for (int i = threadIdx.x; i < (kcap + 1) * C; i += blockDim.x) {
    const int k = i / C, cc = i % C;
    dbl[i] = k >= 1 ? (double)a.db[(size_t)(k < K - 1 ? k : K - 1) * C + cc] : kDNegInf;
  }
  __syncthreads();
  const int b = blockIdx.x * wpb + warp;
  if (warp >= wpb || b >= a.B) return;
  // E of the last R positions, each held twice (slots s and s + R of [2R][C])
  // so that positions t-1 .. t-KM are at fixed offsets below slot
  // (t mod R) + R; slots never written hold -inf.
  double* ring = vsm + (size_t)(kcap + 1) * C + (size_t)warp * 2 * R * C;
  // the label argmax of the same positions (for the packed backpointer)
  uint8_t* rarg = reinterpret_cast<uint8_t*>(vsm + (size_t)(kcap + 1) * C +
                                             (size_t)wpb * 2 * R * C) + (size_t)warp * R * C;
  for (int i = lane; i < 2 * R * C; i += 32) ring[i] = kDNegInf;
  __syncwarp();
  const int c = HALF ? (lane & 15) : lane;
  const int hf = HALF ? lane >> 4 : 0;  // which half of the candidates
  const bool cv = c < C;
  const bool wr = cv && hf == 0;        // the lane that writes label c's outputs
  const int Rm = R - 1;
  const long long lraw = a.lengths[b];
  const int Lb = lraw < 0 ? 0 : (lraw > T ? T : (int)lraw);
  const float* cum_b = a.cum + (size_t)b * (T + 1) * C;
  int16_t* bpk_b = a.bp_k ? a.bp_k + (size_t)b * (T + 1) * C : nullptr;
  uint8_t* bpc_b = a.bp_c ? a.bp_c + (size_t)b * (T + 1) * C : nullptr;
  uint16_t* bp_b = a.bp ? a.bp + (size_t)b * (T + 1) * C : nullptr;

  // this lane's sources q = hf*NQ + j of column c of the transition matrix,
  // -inf beyond C
  double trc[NQ];
#pragma unroll
  for (int j = 0; j < NQ; ++j) {
    const int q = hf * NQ + j;
    trc[j] = (cv && q < C) ? (double)a.tr[(size_t)q * C + c] : kDNegInf;
  }
  // this lane's durations k = hf*KH + j (j = 1 .. KH) of label c's bias row,
  // -inf outside 1 .. kcap
  double dbr[kDbReg ? KH + 1 : 1];
#pragma unroll
  for (int j = 0; j < (kDbReg ? KH + 1 : 1); ++j) {
    const int k = hf * KH + j;
    dbr[j] = (kDbReg && cv && j >= 1 && k <= kcap) ? dbl[k * C + c] : kDNegInf;
  }
  // the two halves' maxima joined: the lower half (smaller index) wins ties
  auto join = [&](double& v, int& ix) {
    if (HALF) {
      const double ov = __shfl_xor_sync(0xffffffffu, v, 16);
      const int oi = __shfl_xor_sync(0xffffffffu, ix, 16);
      if (hf == 0 ? ov > v : ov >= v) {
        v = ov;
        ix = oi;
      }
    }
  };

  // m = max_q (x_q + tr[q,c]) and its first maximiser (x of label q is in lane q)
  auto label_max = [&](double x, int& arg) -> double {
    double v[NQ];
    int ix[NQ];
#pragma unroll
    for (int j = 0; j < NQ; ++j) {
      v[j] = __shfl_sync(0xffffffffu, x, hf * NQ + j) + trc[j];
      ix[j] = hf * NQ + j;
    }
    stable_max<NQ>(v, ix);
    join(v[0], ix[0]);
    arg = ix[0];
    return v[0];
  };

  // position 0: x = 0 for every label
  int arg = 0;
  double x = 0.0;
  {
    const double m = label_max(cv ? 0.0 : kDNegInf, arg);
    if (wr) {
      const double ps = (a.ps && T > 0) ? (double)a.ps[(size_t)b * T * C + c] : 0.0;
      ring[c] = ring[(size_t)R * C + c] = (m + ps) - (double)cum_b[c];
      rarg[c] = (uint8_t)arg;
      if (bpc_b) bpc_b[c] = (uint8_t)arg;
    }
  }
  // cum rows t+1 .. t+4 in flight: a global load's latency spans several steps
  float q0 = (cv && Lb >= 1) ? cum_b[(size_t)1 * C + c] : 0.f;
  float q1 = (cv && Lb >= 2) ? cum_b[(size_t)2 * C + c] : 0.f;
  float q2 = (cv && Lb >= 3) ? cum_b[(size_t)3 * C + c] : 0.f;
  float q3 = (cv && Lb >= 4) ? cum_b[(size_t)4 * C + c] : 0.f;
  for (int t = 1; t <= Lb; ++t) {
    const double cum_t = (double)q0;
    q0 = q1;
    q1 = q2;
    q2 = q3;
    if (t + 4 <= Lb && cv) q3 = cum_b[(size_t)(t + 4) * C + c];
    double best = kDNegInf;
    int bk = 0;
    if (cv) {
      // durations past K-1 have a -inf bias and positions before 0 a -inf
      // source, so the scan needs no bounds
      const double* top = ring + ((size_t)(t & Rm) + R) * C + c;
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        double v[KG];
        int ix[KG];
#pragma unroll
        for (int j = 0; j < KG; ++j) {
          const int kl = g * KG + j + 1;  // this lane's duration index
          const int k = hf * KH + kl;
          const double db_k = kDbReg ? dbr[kl] : (k <= kcap ? dbl[k * C + c] : kDNegInf);
          v[j] = top[-k * C] + db_k;
          ix[j] = k;
        }
        stable_max<KG>(v, ix);
        if (v[0] > best) {  // groups in k order: ties keep the earlier group
          best = v[0];
          bk = ix[0];
        }
      }
    }
    join(best, bk);
    if (best != kDNegInf) best += cum_t;
    x = best;
    if (cv && best != kDNegInf && a.pe) x = best + (double)a.pe[((size_t)b * T + t - 1) * C + c];
    if (wr && bpk_b) bpk_b[(size_t)t * C + c] = (int16_t)bk;
    if (wr && bp_b) {
      // duration in the low byte, the source label at the segment start above
      const int src = bk > 0 ? rarg[((t - bk) & Rm) * C + c] : 0;
      bp_b[(size_t)t * C + c] = (uint16_t)(bk | (src << 8));
    }
    const double m = label_max(cv ? x : kDNegInf, arg);
    if (wr) {
      const double ps = (a.ps && t < T) ? (double)a.ps[((size_t)b * T + t) * C + c] : 0.0;
      const double ne = (m + ps) - cum_t;
      ring[(size_t)(t & Rm) * C + c] = ne;
      ring[((size_t)(t & Rm) + R) * C + c] = ne;
      rarg[(t & Rm) * C + c] = (uint8_t)arg;
      if (bpc_b) bpc_b[(size_t)t * C + c] = (uint8_t)arg;
    }
  }
  // score = max_c x[Lb,c] and the first maximising label
  double mv = wr ? x : kDNegInf;
  if (Lb == 0) mv = wr ? 0.0 : kDNegInf;
  double mx = mv;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  int cand = (wr && mv == mx) ? c : 0x7fffffff;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cand = min(cand, __shfl_xor_sync(0xffffffffu, cand, o));
  if (lane == 0) {
    const double sc = (Lb == 0 || mx == kDNegInf) ? (double)kRefNegInf : mx;
    if (a.partition) a.partition[b] = (float)sc;
    if (a.logz) a.logz[b] = sc;
    if (a.final_c) a.final_c[b] = (cand == 0x7fffffff) ? 0 : cand;
  }
}

template <int NC>
cudaError_t launch_nc(const VChainArgs& a, const VPlan& p, cudaStream_t s) {
  auto go = [&](auto kern) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)p.smem + 8);
    if (e != cudaSuccess) return e;
    kern<<<(a.B + p.wpb - 1) / p.wpb, 32 * p.wpb, p.smem + 8, s>>>(a, p.kcap, p.R, p.wpb);
    return cudaGetLastError();
  };
  if (p.kcap <= 16) return go(vchain_kernel<NC, 16>);
  if (p.kcap <= 32) return go(vchain_kernel<NC, 32>);
  return go(vchain_kernel<NC, 64>);
}

}  // namespace

bool vchain_supported(int B, int C, int K) {
  VPlan p;
  return vplan(p, B, C, K);
}

cudaError_t launch_vchain(const VChainArgs& a, cudaStream_t s) {
  if (a.B <= 0) return cudaSuccess;
  VPlan p;
  if (!vplan(p, a.B, a.C, a.K)) return cudaErrorInvalidValue;
  if (a.C <= 8) return launch_nc<8>(a, p, s);
  if (a.C <= 16) return launch_nc<16>(a, p, s);
  return launch_nc<32>(a, p, s);
}

}  // namespace semicrf
