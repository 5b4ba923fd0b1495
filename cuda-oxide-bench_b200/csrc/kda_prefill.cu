// kda_prefill.cu — KDA (per-channel gate) prefill over T tokens, recurrent
// form with the state held on chip for the whole sequence.
//
// The reference defines KDA only as the per-token step naive_recurrent_kda_step
// (analysis/wave15-attention-architecture/reference/pytorch_reference_kda.py:42-71,
// duplicated in cutile-attn-kda/main.py:147-179); prefill is T applications of
// it, the state threaded from one token to the next:
//   S   = diag(exp(g_t)) S
//   r   = v_t - S^T k_t
//   S  += beta_t k_t r^T
//   o_t = (scale q_t)^T S
// evaluated in fp32 in a rescaled basis so that the per-token decay costs
// nothing per state element.  Within a segment of tokens the state is kept as
// S = diag(c) S~, c the per-row product of exp(g) since the segment start:
//   u   = (k . c)^T S~,      p = (scale q . c)^T S~,     r = v - u
//   S~ += (beta k / c) r^T,  o = p + beta (scale q . k) r
// which is the reference step up to rounding.  A segment starts at every
// 16-token chunk and wherever some row's c would leave [2^-64, 2^64]; there the
// state is renormalised (S~ <- diag(c_prev exp(g_t)) S~, c = 1), which keeps
// 1/c finite for any gate values (a gate that underflows exp() simply zeroes
// the row, as the reference does).
//
// Work split: one CTA per (batch, value head, 64-column slab of d_v), 8 warps
// of 8 state columns each.  Lane l owns d_k / 32 distinct rows of its warp's
// 8 columns (as packed row pairs; the f32x2 instructions handle two rows at a
// time), so each token's vectors are read once per warp without bank
// conflicts.  Each lane's column slots are permuted by its lane bits, which
// lets a 16-shuffle reduce-scatter finish the 16 column sums (k and q for 8
// columns) without selects; 8 more shuffles broadcast the rank-1 coefficients.
// Per 16-token chunk the CTA stages q, k, g, v and beta with cp.async
// (double-buffered: the next chunk is in flight while this one computes),
// forms the rescaled vectors once per row, and writes the chunk's outputs with
// 16-byte stores.
//
// Bound: three fp32 FMAs per state element and token (two column sums and
// the rank-1 update) on the CUDA cores; HBM traffic is only the inputs and
// outputs.  The chunked tensor-core form (per-channel gate inside the WY
// transform) is the faster successor.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "common.cuh"
#include "ptx.cuh"

namespace gdn {
namespace kda_prefill {

constexpr int kBV = 64;                        // state columns per CTA
constexpr int kComputeWarps = kBV / 8;         // each compute warp owns 8 columns
constexpr int kConvWarps = 4;                  // stage and convert the next chunk
constexpr int kComputeThreads = kComputeWarps * 32;
constexpr int kConvThreads = kConvWarps * 32;
constexpr int kThreads = kComputeThreads + kConvThreads;  // 384
constexpr int kTC = 16;                        // tokens per chunk
// named barriers: chunk buffer b full (converter -> compute) and empty
// (compute -> converter), and the converter warps' own barrier
constexpr int kBarFull = 1, kBarEmpty = 3, kBarConv = 5;

template <int DK>
struct Traits {
  // Lanes l and l ^ 16 share rows; lane l owns rows g*64 + 4*(l & 15) + [0, 4)
  // for g < kG, so each 16-lane half reads every row of a token's vectors once,
  // without bank conflicts (the two halves read the same words: broadcast).
  static constexpr int kG = DK / 64;            // float4 loads per vector
  static constexpr int kR = 4 * kG;             // rows per lane (= d_k / 16)
  static constexpr int kP = kR / 2;             // row pairs per lane
  // raw staging buffer (one): the next chunk's inputs as they lie in HBM
  static constexpr int kRawQ = 0;
  static constexpr int kRawK = kRawQ + kTC * DK * 2;
  static constexpr int kRawG = kRawK + kTC * DK * 2;   // room for fp32 gates
  static constexpr int kRawV = kRawG + kTC * DK * 4;
  static constexpr int kRawBeta = kRawV + kTC * kBV * 2;
  static constexpr int kRawBytes = kRawBeta + kTC * 4;
  // double-buffered fp32 chunk vectors [2][kTC][DK]: exp(g), overwritten in
  // place by the renormalisation factors; k.c, scale q.c, beta k / c
  static constexpr int kVecBytes = kTC * DK * 4;
  static constexpr int kE = kRawBytes;
  static constexpr int kKC = kE + 2 * kVecBytes;
  static constexpr int kQC = kKC + 2 * kVecBytes;
  static constexpr int kKD = kQC + 2 * kVecBytes;
  static constexpr int kV = kKD + 2 * kVecBytes;       // v [2][kTC][kBV]
  static constexpr int kBQK = kV + 2 * kTC * kBV * 4;  // beta (scale q).k [2][kTC]
  static constexpr int kBeta = kBQK + 2 * kTC * 4;     // converter scratch [kTC]
  static constexpr int kEmin = kBeta + kTC * 4;        // min / max of exp(g) over rows
  static constexpr int kEmax = kEmin + kTC * 4;
  static constexpr int kCarry = kEmax + kTC * 4;       // c per row across chunks
  static constexpr int kMask = kCarry + DK * 4;        // segment starts [2]
  static constexpr int kO = kMask + 16;                // outputs [2][kTC][kBV]
  static constexpr int kSmem = kO + 2 * kTC * kBV * 2;
  static_assert(kRawBytes % 16 == 0 && kE % 16 == 0 && kV % 16 == 0 && kCarry % 16 == 0 &&
                    kO % 16 == 0,
                "16-byte aligned staging");
};

__device__ __forceinline__ void bar_sync_n(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void bar_arrive_n(int id, int n) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic): two state rows per instruction.
__device__ __forceinline__ uint64_t pack2f(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float lo2f(uint64_t v) {
  return __uint_as_float(static_cast<uint32_t>(v));
}
__device__ __forceinline__ float hi2f(uint64_t v) {
  return __uint_as_float(static_cast<uint32_t>(v >> 32));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// A 2-byte shared store that the compiler does not treat as aliasing the
// staged vectors, so the next token's shared loads may move above it (the
// block barriers order it against the flush).
template <typename IO>
__device__ __forceinline__ void sts16(uint32_t addr, IO x) {
  asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr), "h"(*reinterpret_cast<unsigned short*>(&x)));
}

template <typename IO>
__device__ __forceinline__ void unpack8(uint4 w, float* f) {
  const IO* e = reinterpret_cast<const IO*>(&w);
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] = to_f32<IO>(e[j]);
}

#ifdef GDN_PREFILL_TRACE
// Phase timestamps of CTA 0, thread 0 (profiling builds only): [chunk][phase].
__device__ unsigned long long g_kda_trace[64 * 4];
#define KTRACE(c, ph)                                                      \
  do {                                                                     \
    if (blockIdx.x == 0 && threadIdx.x == 0 && (c) < 64)                   \
      g_kda_trace[(c) * 4 + (ph)] = global_timer_ns();                     \
  } while (0)
#else
#define KTRACE(c, ph) \
  do {                \
  } while (0)
#endif

template <int DK, typename IO>
__global__ void __launch_bounds__(kThreads, DK == 256 ? 1 : 2)
    kda_prefill_kernel(const gdn_prefill_args_t a) {
  using Tr = Traits<DK>;
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* raw = smem;
  float* sE = reinterpret_cast<float*>(smem + Tr::kE);
  float* sKC = reinterpret_cast<float*>(smem + Tr::kKC);
  float* sQC = reinterpret_cast<float*>(smem + Tr::kQC);
  float* sKD = reinterpret_cast<float*>(smem + Tr::kKD);
  float* sV = reinterpret_cast<float*>(smem + Tr::kV);
  float* sBQK = reinterpret_cast<float*>(smem + Tr::kBQK);
  float* sBeta = reinterpret_cast<float*>(smem + Tr::kBeta);
  float* sEmin = reinterpret_cast<float*>(smem + Tr::kEmin);
  float* sEmax = reinterpret_cast<float*>(smem + Tr::kEmax);
  float* sCarry = reinterpret_cast<float*>(smem + Tr::kCarry);
  uint32_t* sMask = reinterpret_cast<uint32_t*>(smem + Tr::kMask);
  IO* sO = reinterpret_cast<IO*>(smem + Tr::kO);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nslab = a.dv / kBV;
  const int slab = blockIdx.x % nslab;
  const int bh = blockIdx.x / nslab;
  const int h = bh % a.Hv, b = bh / a.Hv;
  const int col0 = slab * kBV;
  const int T = a.T;
  const int nchunks = (T + kTC - 1) / kTC;
  const int64_t tok_base = static_cast<int64_t>(b) * T;
  constexpr unsigned kFull = 0xffffffffu;

  if (warp >= kComputeWarps) {
    // ------------------------------------------------------------ converter
    // Stages chunk c+1 while the compute warps run chunk c: cp.async loads,
    // exp(g), the segment starts, the rescaled vectors; flushes outputs.
    constexpr float kLo = 5.421010862427522e-20f;  // 2^-64
    constexpr float kHi = 1.8446744073709552e19f;  // 2^64
    const int ct = tid - kComputeThreads, cw = ct >> 5;
    const int hq = h / (a.Hv / a.Hqk);
    const int gsz = a.g_dtype == GDN_DT_F32 ? 4 : 2;
    const int bsz = a.beta_dtype == GDN_DT_F32 ? 4 : 2;
    const IO* q = static_cast<const IO*>(a.q);
    const IO* k = static_cast<const IO*>(a.k);
    const IO* v = static_cast<const IO*>(a.v);
    const unsigned char* g = static_cast<const unsigned char*>(a.g);
    const unsigned char* beta = static_cast<const unsigned char*>(a.beta);
    IO* o = static_cast<IO*>(a.o);

    auto issue = [&](int c) {
      const int t0 = c * kTC, n = min(kTC, T - t0);
      constexpr int qp = DK / 8;  // 16-byte pieces per q/k row
      for (int i = ct; i < n * qp; i += kConvThreads) {
        const int t = i / qp, p = i % qp;
        const int64_t off = ((tok_base + t0 + t) * a.Hqk + hq) * DK + p * 8;
        cp_async16(raw + Tr::kRawQ + (t * DK + p * 8) * 2, q + off);
        cp_async16(raw + Tr::kRawK + (t * DK + p * 8) * 2, k + off);
      }
      const int gp = DK * gsz / 16;
      for (int i = ct; i < n * gp; i += kConvThreads) {
        const int t = i / gp, p = i % gp;
        const int64_t off = ((tok_base + t0 + t) * a.Hv + h) * DK * gsz + p * 16;
        cp_async16(raw + Tr::kRawG + t * DK * gsz + p * 16, g + off);
      }
      constexpr int vp = kBV * 2 / 16;
      for (int i = ct; i < n * vp; i += kConvThreads) {
        const int t = i / vp, p = i % vp;
        const int64_t off = ((tok_base + t0 + t) * a.Hv + h) * a.dv + col0 + p * 8;
        cp_async16(raw + Tr::kRawV + (t * kBV + p * 8) * 2, v + off);
      }
      if (ct < n) {
        // the aligned 32-bit word holding this token's beta (beta is 4-byte
        // aligned).  For a 2-byte beta in the low half of its word, the word
        // reaches 2 bytes past the element; for the tensor's last element that
        // is past its end, so that one element is read with a 2-byte load.
        const int64_t bi = (tok_base + t0 + ct) * a.Hv + h;
        const uintptr_t e = reinterpret_cast<uintptr_t>(beta + bi * bsz);
        if (bsz == 2 && (e & 2) == 0 && bi == static_cast<int64_t>(a.B) * a.T * a.Hv - 1)
          *reinterpret_cast<unsigned short*>(raw + Tr::kRawBeta + ct * 4) =
              *reinterpret_cast<const unsigned short*>(e);
        else
          cp_async4(raw + Tr::kRawBeta + ct * 4, reinterpret_cast<const void*>(e & ~uintptr_t(3)));
      }
      cp_async_commit();
    };
    auto flush = [&](int c) {
      const int t0 = c * kTC, n = min(kTC, T - t0);
      const IO* src = sO + (c & 1) * kTC * kBV;
      constexpr int op = kBV * 2 / 16;
      for (int i = ct; i < n * op; i += kConvThreads) {
        const int t = i / op, p = i % op;
        const int64_t off = ((tok_base + t0 + t) * a.Hv + h) * a.dv + col0 + p * 8;
        *reinterpret_cast<uint4*>(o + off) = *reinterpret_cast<const uint4*>(src + t * kBV + p * 8);
      }
    };

    for (int r = ct; r < DK; r += kConvThreads) sCarry[r] = 1.f;
    issue(0);
    for (int c = 0; c < nchunks; ++c) {
      const int bs = c & 1;
      const int t0 = c * kTC, n = min(kTC, T - t0);
      float* E = sE + bs * kTC * DK;
      float* KC = sKC + bs * kTC * DK;
      float* QC = sQC + bs * kTC * DK;
      float* KD = sKD + bs * kTC * DK;
      float* V = sV + bs * kTC * kBV;
      float* BQK = sBQK + bs * kTC;
      const IO* rq = reinterpret_cast<const IO*>(raw + Tr::kRawQ);
      const IO* rk = reinterpret_cast<const IO*>(raw + Tr::kRawK);
      cp_async_wait_all();
      bar_sync_n(kBarConv, kConvThreads);  // chunk c staged
      if (c >= 2) {  // buffer bs is free once the compute warps are done with chunk c-2
        bar_sync_n(kBarEmpty + bs, kThreads);
        flush(c - 2);
      }
      for (int i = ct; i < n * (DK / 4); i += kConvThreads) {
        const int t = i / (DK / 4), r = (i % (DK / 4)) * 4;
        const unsigned char* row = raw + Tr::kRawG + t * DK * gsz;
        *reinterpret_cast<float4*>(E + t * DK + r) =
            make_float4(expf(smem_any(row, r, a.g_dtype)), expf(smem_any(row, r + 1, a.g_dtype)),
                        expf(smem_any(row, r + 2, a.g_dtype)),
                        expf(smem_any(row, r + 3, a.g_dtype)));
      }
      for (int i = ct; i < n * (kBV / 8); i += kConvThreads) {
        const int t = i / (kBV / 8), cc = (i % (kBV / 8)) * 8;
        float f[8];
        unpack8<IO>(*reinterpret_cast<const uint4*>(raw + Tr::kRawV + (t * kBV + cc) * 2), f);
        *reinterpret_cast<float4*>(V + t * kBV + cc) = make_float4(f[0], f[1], f[2], f[3]);
        *reinterpret_cast<float4*>(V + t * kBV + cc + 4) = make_float4(f[4], f[5], f[6], f[7]);
      }
      if (ct < n) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(raw + Tr::kRawBeta + ct * 4);
        float bt;
        if (a.beta_dtype == GDN_DT_F32) {
          bt = __uint_as_float(w);
        } else {
          const uintptr_t e =
              reinterpret_cast<uintptr_t>(beta + ((tok_base + t0 + ct) * a.Hv + h) * bsz);
          const unsigned short r16 =
              static_cast<unsigned short>((e & 2) ? (w >> 16) : (w & 0xFFFFu));
          bt = a.beta_dtype == GDN_DT_BF16 ? __uint_as_float(static_cast<uint32_t>(r16) << 16)
                                           : __half2float(__ushort_as_half(r16));
        }
        sBeta[ct] = bt;
      }
      bar_sync_n(kBarConv, kConvThreads);
      // per token: beta (scale q).k, and the smallest / largest exp(g) over rows
      for (int t = cw; t < n; t += kConvWarps) {
        float d = 0.f, mn = INFINITY, mx = 0.f;
#pragma unroll
        for (int j = lane; j < DK; j += 32) {
          d = fmaf(to_f32<IO>(rq[t * DK + j]), to_f32<IO>(rk[t * DK + j]), d);
          const float e = E[t * DK + j];
          mn = fminf(mn, e);
          mx = fmaxf(mx, e);
        }
#pragma unroll
        for (int m = 16; m; m >>= 1) {
          d += __shfl_xor_sync(kFull, d, m);
          mn = fminf(mn, __shfl_xor_sync(kFull, mn, m));
          mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, m));
        }
        if (lane == 0) {
          BQK[t] = sBeta[t] * d * a.scale;
          sEmin[t] = mn;
          sEmax[t] = mx;
        }
      }
      bar_sync_n(kBarConv, kConvThreads);
      // Segment starts: every chunk start, and wherever the product of the
      // per-token extremes could take some row's c out of [2^-64, 2^64]
      // (conservative: bounds every row at once).
      if (ct == 0) {
        uint32_t m = 1u;
        float lo = 1.f, hi = 1.f;
        for (int t = 1; t < n; ++t) {
          lo *= sEmin[t];
          hi *= sEmax[t];
          if (!(lo >= kLo && hi <= kHi)) {
            m |= 1u << t;
            lo = 1.f;
            hi = 1.f;
          }
        }
        sMask[bs] = m;
      }
      bar_sync_n(kBarConv, kConvThreads);
      const uint32_t mask = sMask[bs];
      for (int r = ct; r < DK; r += kConvThreads) {
        float e[kTC], kf[kTC], qf[kTC];
#pragma unroll
        for (int t = 0; t < kTC; ++t)
          if (t < n) {
            e[t] = E[t * DK + r];
            kf[t] = to_f32<IO>(rk[t * DK + r]);
            qf[t] = to_f32<IO>(rq[t * DK + r]) * a.scale;
          }
        float cc = sCarry[r];
#pragma unroll
        for (int t = 0; t < kTC; ++t)
          if (t < n) {
            if ((mask >> t) & 1u) {
              E[t * DK + r] = cc * e[t];  // renormalisation factor before token t
              cc = 1.f;
            } else {
              cc *= e[t];
            }
            KC[t * DK + r] = kf[t] * cc;
            QC[t * DK + r] = qf[t] * cc;
            KD[t * DK + r] = sBeta[t] * kf[t] * __frcp_rn(cc);
          }
        sCarry[r] = cc;
      }
      __threadfence_block();
      bar_sync_n(kBarConv, kConvThreads);  // raw fully read, vectors written
      if (c + 1 < nchunks) issue(c + 1);
      bar_arrive_n(kBarFull + bs, kThreads);
    }
    for (int c = max(0, nchunks - 2); c < nchunks; ++c) {
      bar_sync_n(kBarEmpty + (c & 1), kThreads);
      flush(c);
    }
    return;
  }

  // -------------------------------------------------------------- compute
  // Lane geometry.  Half hf = lane >> 4 of the warp owns state columns
  // warp*8 + hf*4 + [0, 4); lane slot cc holds column warp*8 + hf*4 +
  // (cc ^ perm) at the lane's kR rows, packed as row pairs s2[p][cc].  After
  // the reduce-scatter over the 16 lanes of a half, lane l holds the full sum
  // of slot 0 (column ... + perm): k^T S when bit 3 of l is clear, (scale q)^T S
  // when it is set (those lanes accumulate the q sums in the k slots).
  const int hf = lane >> 4;
  const int perm = (lane >> 1) & 3;
  const int colw = warp * 8 + hf * 4 + perm;
  const bool qlane = lane & 8;
  const bool o_lane = qlane && !(lane & 1);
  const int lr = lane & 15;
  auto row_of = [&](int p, int half) { return (p >> 1) * 64 + 4 * lr + 2 * (p & 1) + half; };
  auto load_pairs = [&](const float* base, uint64_t* out) {
#pragma unroll
    for (int gi = 0; gi < Tr::kG; ++gi) {
      const float4 x = lds128(base + gi * 64 + 4 * lr);
      out[2 * gi] = pack2f(x.x, x.y);
      out[2 * gi + 1] = pack2f(x.z, x.w);
    }
  };

  uint64_t s2[Tr::kP][4];
  const int64_t sbase = static_cast<int64_t>(bh) * DK * a.dv + col0 + warp * 8 + hf * 4;
  if (a.initial_state) {
    const float* S0 = a.initial_state + sbase;
#pragma unroll
    for (int p = 0; p < Tr::kP; ++p) {
      const float* r0 = S0 + static_cast<int64_t>(row_of(p, 0)) * a.dv;
      const float* r1 = S0 + static_cast<int64_t>(row_of(p, 1)) * a.dv;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc)
        s2[p][cc] = pack2f(__ldg(r0 + (cc ^ perm)), __ldg(r1 + (cc ^ perm)));
    }
  } else {
#pragma unroll
    for (int p = 0; p < Tr::kP; ++p)
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) s2[p][cc] = 0;
  }
  // source lane of the rank-1 coefficient of slot cc (a k lane of this half)
  int bsrc[4];
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) bsrc[cc] = (lane & 16) | ((cc ^ perm) << 1);

  for (int c = 0; c < nchunks; ++c) {
    const int bs = c & 1;
    bar_sync_n(kBarFull + bs, kThreads);
    KTRACE(c, 0);
    const uint32_t mask = sMask[bs];
    const int n = min(kTC, T - c * kTC);
    const float* E = sE + bs * kTC * DK;
    const float* A = (qlane ? sQC : sKC) + bs * kTC * DK;
    const float* Bv = (qlane ? sKC : sQC) + bs * kTC * DK;
    const float* KD = sKD + bs * kTC * DK;
    const float* V = sV + bs * kTC * kBV;
    const float* BQK = sBQK + bs * kTC;
    const uint32_t o_addr0 = smem_u32(sO + bs * kTC * kBV + colw);
    // fully unrolled: every per-token offset and mask bit becomes an immediate
#pragma unroll
    for (int t = 0; t < kTC; ++t) {
      if (t >= n) break;
      if ((mask >> t) & 1u) {  // segment start: S~ <- diag(R) S~
        uint64_t r2[Tr::kP];
        load_pairs(E + t * DK, r2);
#pragma unroll
        for (int p = 0; p < Tr::kP; ++p)
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) s2[p][cc] = mul2(s2[p][cc], r2[p]);
      }
      uint64_t A2[Tr::kP], B2[Tr::kP], D2[Tr::kP];
      load_pairs(A + t * DK, A2);
      load_pairs(Bv + t * DK, B2);
      load_pairs(KD + t * DK, D2);
      float v8[8];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint64_t u2 = mul2(A2[0], s2[0][cc]), p2 = mul2(B2[0], s2[0][cc]);
#pragma unroll
        for (int p = 1; p < Tr::kP; ++p) {
          u2 = fma2(A2[p], s2[p][cc], u2);
          p2 = fma2(B2[p], s2[p][cc], p2);
        }
        v8[cc] = lo2f(u2) + hi2f(u2);
        v8[4 + cc] = lo2f(p2) + hi2f(p2);
      }
      // reduce-scatter over the 16 lanes of this half: no selects, thanks to
      // the slot permutation (partners hold the matching column in the sent slots)
      float w4[4], w2[2];
#pragma unroll
      for (int i = 0; i < 4; ++i) w4[i] = v8[i] + __shfl_xor_sync(kFull, v8[i + 4], 8);
#pragma unroll
      for (int i = 0; i < 2; ++i) w2[i] = w4[i] + __shfl_xor_sync(kFull, w4[i + 2], 4);
      float z = w2[0] + __shfl_xor_sync(kFull, w2[1], 2);
      z += __shfl_xor_sync(kFull, z, 1);
      // r = v - k^T S (k lanes), shared with the q lane of the same column
      const float r = V[t * kBV + colw] - z;
      const float rx = __shfl_sync(kFull, r, lane & ~8);
      if (o_lane) sts16(o_addr0 + t * kBV * 2, from_f32<IO>(fmaf(BQK[t], rx, z)));
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const float bc = __shfl_sync(kFull, rx, bsrc[cc]);
        const uint64_t b2 = pack2f(bc, bc);
#pragma unroll
        for (int p = 0; p < Tr::kP; ++p) s2[p][cc] = fma2(D2[p], b2, s2[p][cc]);
      }
    }
    KTRACE(c, 1);
    __threadfence_block();
    bar_arrive_n(kBarEmpty + bs, kThreads);
  }
  // S = diag(c) S~ (the converter's last carry update preceded the final
  // chunk's hand-off)
  uint64_t c2[Tr::kP];
  load_pairs(sCarry, c2);
  float* S1 = a.final_state + sbase;
#pragma unroll
  for (int p = 0; p < Tr::kP; ++p) {
    float* r0 = S1 + static_cast<int64_t>(row_of(p, 0)) * a.dv;
    float* r1 = S1 + static_cast<int64_t>(row_of(p, 1)) * a.dv;
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      const uint64_t x = mul2(s2[p][cc], c2[p]);
      r0[cc ^ perm] = lo2f(x);
      r1[cc ^ perm] = hi2f(x);
    }
  }
}

int validate(const gdn_prefill_args_t* a) {
  if (!a) return GDN_ERR_NULL;
  if (!a->q || !a->k || !a->v || !a->g || !a->beta || !a->final_state || !a->o) return GDN_ERR_NULL;
  if (a->B < 1 || a->T < 1 || a->Hqk < 1 || a->Hv < 1 || a->Hv % a->Hqk) return GDN_ERR_SHAPE;
  if (a->dk != 64 && a->dk != 128 && a->dk != 256) return GDN_ERR_SHAPE;
  if (a->dv != 64 && a->dv != 128 && a->dv != 256) return GDN_ERR_SHAPE;
  if (static_cast<int64_t>(a->B) * a->Hv * (a->dv / kBV) > 0x7FFFFFFF) return GDN_ERR_SHAPE;
  if (static_cast<int64_t>(a->B) * a->T > 0x7FFFFFFF) return GDN_ERR_SHAPE;
  if (a->io_dtype != GDN_DT_BF16 && a->io_dtype != GDN_DT_F16) return GDN_ERR_DTYPE;
  if (!dtype_valid(a->g_dtype) || !dtype_valid(a->beta_dtype)) return GDN_ERR_DTYPE;
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->o) ||
      !aligned16(a->g) || (reinterpret_cast<uintptr_t>(a->beta) & 3) ||
      (reinterpret_cast<uintptr_t>(a->final_state) & 3) ||
      (reinterpret_cast<uintptr_t>(a->initial_state) & 3))
    return GDN_ERR_ALIGN;
  return GDN_OK;
}

template <int DK, typename IO>
int launch_dk(const gdn_prefill_args_t& a, cudaStream_t stream) {
  static std::atomic<uint64_t> attr_done{0};
  auto kern = kda_prefill_kernel<DK, IO>;
  int rc = ensure_smem_attr(kern, Traits<DK>::kSmem, attr_done);
  if (rc) return rc;
  const unsigned grid = static_cast<unsigned>(static_cast<int64_t>(a.B) * a.Hv * (a.dv / kBV));
  kern<<<grid, kThreads, Traits<DK>::kSmem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

template <typename IO>
int launch(const gdn_prefill_args_t& a, cudaStream_t stream) {
  switch (a.dk) {
    case 64: return launch_dk<64, IO>(a, stream);
    case 128: return launch_dk<128, IO>(a, stream);
    default: return launch_dk<256, IO>(a, stream);
  }
}

}  // namespace kda_prefill
}  // namespace gdn

#ifdef GDN_PREFILL_TRACE
extern "C" int kda_prefill_trace_read(unsigned long long* host) {
  return cudaMemcpyFromSymbol(host, gdn::kda_prefill::g_kda_trace,
                              sizeof(gdn::kda_prefill::g_kda_trace)) == cudaSuccess
             ? 0
             : 1;
}
#endif

namespace gdn {
namespace prefill {
int kda_chunked_launch(const gdn_prefill_args_t& a, cudaStream_t stream);  // gdn_prefill.cu
}
}  // namespace gdn

extern "C" int kda_prefill_launch(const gdn_prefill_args_t* args, gdn_stream_t stream) {
  int rc = gdn::kda_prefill::validate(args);
  if (rc) return rc;
  gdn::DeviceInfo di;
  if ((rc = gdn::device_info(&di))) return rc;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  // chunked tensor-core form when the caller passes a workspace (d = 128)
  if (args->workspace) return gdn::prefill::kda_chunked_launch(*args, s);
  return args->io_dtype == GDN_DT_BF16 ? gdn::kda_prefill::launch<__nv_bfloat16>(*args, s)
                                       : gdn::kda_prefill::launch<__half>(*args, s);
}
