// vchain.cu -- max-semiring chain for C <= 32: one warp per sequence.
//
// Reference semantics: the max branch of streaming/pytorch_reference.py:
// 116-273 (forward) with the Viterbi backpointers of nn.py:444-505.  The
// factorised recurrence (exact in the max semiring):
//     x[t,c]  = pe[t-1,c] + max_{k=1..min(K',t)} ( (cum[t,c] - cum[t-k,c]) + sv[t-k,c] + db[min(k,K-1),c] )
//     m[s,c]  = max_c' ( x[s,c'] + tr[c',c] ),      sv[s,c] = m[s,c] + ps[s,c]
// with x[0,c] = 0, K' = max(1, K-1), ties to the smallest k (strict >,
// nn.py:494) and to the first c' (nn.py:491); the score is max_c x[L,c] with
// the first maximising label (nn.py:501).  Float32 throughout, as the
// reference computes it, with the content difference taken first as the
// reference's edge does (pytorch_reference.py:87-92).
//
// Lane c of the warp owns label c.  Its source values and cum values of the
// last K' positions live in a per-warp shared-memory ring that only that
// lane reads and writes, so the recurrence needs no barrier; the label
// maximum m is 32 shuffles and a stable argmax tree.  Several sequences run
// per CTA, one per warp, so a batch of B sequences is B warps across the GPU.

#include "semicrf_internal.cuh"

namespace semicrf {

namespace {

constexpr int kVMaxWarps = 4;
constexpr size_t kVSmemMax = 200 * 1024;

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
  const size_t shared = 4 * (size_t)(p.kcap + 1) * C;  // duration bias table
  const size_t per_warp = 17 * (size_t)p.R * C;        // (sv, cum) ring (twice) + argmax ring
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

// NC: labels rounded up to 8/16/32 (the lanes that take part in the label
// maximum).  KM: durations rounded up to 8/16/32/64, with the duration-bias
// row held in registers and the k-scan unrolled.
template <int NC, int KM>
__global__ void __launch_bounds__(32 * kVMaxWarps) vchain_kernel(const VChainArgs a, int kcap,
                                                                 int R, int wpb) {
  extern __shared__ __align__(16) float vsm[];
  const int C = a.C, K = a.K, T = a.T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* dbl = vsm;  // [kcap + 1][C], row k = db[min(k, K-1)]
  for (int i = threadIdx.x; i < (kcap + 1) * C; i += blockDim.x) {
    const int k = i / C, cc = i % C;
    dbl[i] = k >= 1 ? a.db[(size_t)(k < K - 1 ? k : K - 1) * C + cc] : kNegInf;
  }
  __syncthreads();
  const int b = blockIdx.x * wpb + warp;
  if (warp >= wpb || b >= a.B) return;
  // (sv, cum) of the last R positions, each held twice (slots s and s + R of
  // [2R][C] float2) so that positions t-1 .. t-KM are at fixed offsets below
  // slot (t mod R) + R; slots never written hold (-inf, 0).
  const size_t dbl_floats = ((size_t)(kcap + 1) * C + 1) & ~size_t(1);
  float2* ring = reinterpret_cast<float2*>(vsm + dbl_floats) + (size_t)warp * 2 * R * C;
  // the label argmax of the same positions (for the packed backpointer)
  uint8_t* rarg = reinterpret_cast<uint8_t*>(reinterpret_cast<float2*>(vsm + dbl_floats) +
                                             (size_t)wpb * 2 * R * C) + (size_t)warp * R * C;
  for (int i = lane; i < 2 * R * C; i += 32) ring[i] = make_float2(kNegInf, 0.f);
  __syncwarp();
  const int c = lane;
  const bool cv = c < C;
  const int Rm = R - 1;
  const long long lraw = a.lengths[b];
  const int Lb = lraw < 0 ? 0 : (lraw > T ? T : (int)lraw);
  const float* cum_b = a.cum + (size_t)b * (T + 1) * C;
  int16_t* bpk_b = a.bp_k ? a.bp_k + (size_t)b * (T + 1) * C : nullptr;
  uint8_t* bpc_b = a.bp_c ? a.bp_c + (size_t)b * (T + 1) * C : nullptr;
  uint16_t* bp_b = a.bp ? a.bp + (size_t)b * (T + 1) * C : nullptr;

  // column c of the transition matrix (sources q), -inf beyond C
  float trc[NC];
#pragma unroll
  for (int q = 0; q < NC; ++q) trc[q] = (cv && q < C) ? a.tr[(size_t)q * C + c] : kNegInf;
  // duration-bias row of label c in registers (KM > 0)
  float dbr[KM + 1];
#pragma unroll
  for (int k = 0; k <= KM; ++k) dbr[k] = (cv && k >= 1 && k <= kcap) ? dbl[k * C + c] : kNegInf;

  // m = max_q (x_q + tr[q,c]) and its first maximiser
  auto label_max = [&](float x, int& arg) -> float {
    float v[NC];
    int ix[NC];
#pragma unroll
    for (int q = 0; q < NC; ++q) {
      v[q] = __shfl_sync(0xffffffffu, x, q) + trc[q];
      ix[q] = q;
    }
#pragma unroll
    for (int w = 1; w < NC; w <<= 1)
#pragma unroll
      for (int q = 0; q < NC; q += 2 * w)
        if (v[q + w] > v[q]) {  // strict: ties keep the lower index
          v[q] = v[q + w];
          ix[q] = ix[q + w];
        }
    arg = ix[0];
    return v[0];
  };

  // position 0: x = 0 for every label
  int arg = 0;
  float x = 0.f;
  {
    const float m = label_max(cv ? 0.f : kNegInf, arg);
    if (cv) {
      const float ps = (a.ps && T > 0) ? a.ps[(size_t)b * T * C + c] : 0.f;
      ring[c] = ring[(size_t)R * C + c] = make_float2(m + ps, cum_b[c]);
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
    const float cum_t = q0;
    q0 = q1;
    q1 = q2;
    q2 = q3;
    if (t + 4 <= Lb && cv) q3 = cum_b[(size_t)(t + 4) * C + c];
    float best = kNegInf;
    int bk = 0;
    if (cv) {
      // durations past K-1 have a -inf bias and positions before 0 a -inf
      // source, so the scan needs no bounds
      const float2* top = ring + ((size_t)(t & Rm) + R) * C + c;
      float2 e[KM + 1];
#pragma unroll
      for (int k = 1; k <= KM; ++k) e[k] = top[-k * C];
#pragma unroll
      for (int k = 1; k <= KM; ++k) {
        const float v = (cum_t - e[k].y) + e[k].x + dbr[k];
        if (v > best) {  // strict: ties keep the smaller k
          best = v;
          bk = k;
        }
      }
    }
    x = best;
    if (cv && best != kNegInf && a.pe) x = best + a.pe[((size_t)b * T + t - 1) * C + c];
    if (cv && bpk_b) bpk_b[(size_t)t * C + c] = (int16_t)bk;
    if (cv && bp_b) {
      // duration in the low byte, the source label at the segment start above
      const int src = bk > 0 ? rarg[((t - bk) & Rm) * C + c] : 0;
      bp_b[(size_t)t * C + c] = (uint16_t)(bk | (src << 8));
    }
    const float m = label_max(cv ? x : kNegInf, arg);
    if (cv) {
      const float ps = (a.ps && t < T) ? a.ps[((size_t)b * T + t) * C + c] : 0.f;
      const float2 ne = make_float2(m + ps, cum_t);
      ring[(size_t)(t & Rm) * C + c] = ne;
      ring[((size_t)(t & Rm) + R) * C + c] = ne;
      rarg[(t & Rm) * C + c] = (uint8_t)arg;
      if (bpc_b) bpc_b[(size_t)t * C + c] = (uint8_t)arg;
    }
  }
  // score = max_c x[Lb,c] and the first maximising label
  float mv = cv ? x : kNegInf;
  if (Lb == 0) mv = cv ? 0.f : kNegInf;
  float mx = mv;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  int cand = (cv && mv == mx) ? c : 0x7fffffff;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cand = min(cand, __shfl_xor_sync(0xffffffffu, cand, o));
  if (lane == 0) {
    const double sc = (Lb == 0 || mx == kNegInf) ? (double)kRefNegInf : (double)mx;
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
  if (p.kcap <= 8) return go(vchain_kernel<NC, 8>);
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
