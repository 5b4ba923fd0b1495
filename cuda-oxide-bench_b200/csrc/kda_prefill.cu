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
// which this kernel evaluates in fp32 in exactly that order, per token, as
//   p = (scale q)^T S_decayed,  o = p + beta (scale q . k) r
// so the state is read and written once per token from registers, not HBM.
//
// Work split: one CTA per (batch, value head, 64-column slab of d_v), 256
// threads; four threads share one state column, each holding d_k / 4 rows of
// it in registers.  The two column sums per token (k^T S and q^T S) finish
// with two shuffles across those four threads.  Per 16-token chunk the CTA
// stages q, k, g, v and beta with cp.async (double-buffered, the next chunk in
// flight while this one computes), converts them once to fp32 (exp(g), the
// scaled q, q.k) into padded shared vectors that every column thread reads as
// broadcasts, and writes the chunk's outputs with 16-byte stores.
//
// Bound: the recurrent form does 4 d_k d_v fp32 operations per token and head
// (decay, two column sums, rank-1 update) on the CUDA cores; HBM traffic is
// only the inputs and outputs.  The chunked tensor-core form (per-channel gate
// inside the WY transform) is the faster successor.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "common.cuh"
#include "ptx.cuh"

namespace gdn {
namespace kda_prefill {

constexpr int kBV = 64;                  // state columns per CTA
constexpr int kSplit = 4;                // threads per state column
constexpr int kThreads = kBV * kSplit;   // 256
constexpr int kTC = 16;                  // tokens per staged chunk

template <int DK>
struct Traits {
  static constexpr int kRows = DK / kSplit;  // state rows per thread
  static constexpr int kPad = kRows + 4;     // floats per row quarter in a staged vector
  static constexpr int kVec = kSplit * kPad; // floats per staged d_k vector
  // raw staging buffer (two of them): inputs as they lie in HBM
  static constexpr int kRawQ = 0;
  static constexpr int kRawK = kRawQ + kTC * DK * 2;
  static constexpr int kRawG = kRawK + kTC * DK * 2;   // room for fp32 gates
  static constexpr int kRawV = kRawG + kTC * DK * 4;
  static constexpr int kRawBeta = kRawV + kTC * kBV * 2;
  static constexpr int kRawBytes = kRawBeta + kTC * 4;
  // fp32 compute buffers (one) and the bf16/f16 output stage
  static constexpr int kE = 2 * kRawBytes;             // exp(g)
  static constexpr int kK = kE + kTC * kVec * 4;
  static constexpr int kQ = kK + kTC * kVec * 4;       // scale * q
  static constexpr int kV = kQ + kTC * kVec * 4;
  static constexpr int kBeta = kV + kTC * kBV * 4;
  static constexpr int kQK = kBeta + kTC * 4;          // (scale q) . k
  static constexpr int kO = kQK + kTC * 4;
  static constexpr int kSmem = kO + kTC * kBV * 2;
  static_assert(kRawBytes % 16 == 0 && kE % 16 == 0 && kV % 16 == 0 && kO % 16 == 0,
                "16-byte aligned staging");
  static_assert(kRows % 8 == 0, "8-element staging pieces stay inside one row quarter");
};

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

template <typename IO>
__device__ __forceinline__ void unpack8(uint4 w, float* f) {
  const IO* e = reinterpret_cast<const IO*>(&w);
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] = to_f32<IO>(e[j]);
}

template <int DK, typename IO>
__global__ void __launch_bounds__(kThreads, DK == 256 ? 1 : 2)
    kda_prefill_kernel(const gdn_prefill_args_t a) {
  using Tr = Traits<DK>;
  extern __shared__ __align__(128) unsigned char smem[];
  float* sE = reinterpret_cast<float*>(smem + Tr::kE);
  float* sK = reinterpret_cast<float*>(smem + Tr::kK);
  float* sQ = reinterpret_cast<float*>(smem + Tr::kQ);
  float* sV = reinterpret_cast<float*>(smem + Tr::kV);
  float* sBeta = reinterpret_cast<float*>(smem + Tr::kBeta);
  float* sQK = reinterpret_cast<float*>(smem + Tr::kQK);
  IO* sO = reinterpret_cast<IO*>(smem + Tr::kO);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nslab = a.dv / kBV;
  const int slab = blockIdx.x % nslab;
  const int bh = blockIdx.x / nslab;
  const int h = bh % a.Hv, b = bh / a.Hv;
  const int hq = h / (a.Hv / a.Hqk);
  const int col = warp * 8 + (lane & 7);  // state column within the slab
  const int qt = lane >> 3;               // row quarter
  const int col0 = slab * kBV;
  const int T = a.T;
  const int nchunks = (T + kTC - 1) / kTC;
  const int gsz = a.g_dtype == GDN_DT_F32 ? 4 : 2;
  const int bsz = a.beta_dtype == GDN_DT_F32 ? 4 : 2;
  const int64_t tok_base = static_cast<int64_t>(b) * T;

  const IO* q = static_cast<const IO*>(a.q);
  const IO* k = static_cast<const IO*>(a.k);
  const IO* v = static_cast<const IO*>(a.v);
  const unsigned char* g = static_cast<const unsigned char*>(a.g);
  const unsigned char* beta = static_cast<const unsigned char*>(a.beta);
  IO* o = static_cast<IO*>(a.o);

  auto issue = [&](int c) {
    unsigned char* raw = smem + (c & 1) * Tr::kRawBytes;
    const int t0 = c * kTC, n = min(kTC, T - t0);
    constexpr int qp = DK / 8;  // 16-byte pieces per q/k row
    for (int i = tid; i < n * qp; i += kThreads) {
      const int t = i / qp, p = i % qp;
      const int64_t off = ((tok_base + t0 + t) * a.Hqk + hq) * DK + p * 8;
      cp_async16(raw + Tr::kRawQ + (t * DK + p * 8) * 2, q + off);
      cp_async16(raw + Tr::kRawK + (t * DK + p * 8) * 2, k + off);
    }
    const int gp = DK * gsz / 16;
    for (int i = tid; i < n * gp; i += kThreads) {
      const int t = i / gp, p = i % gp;
      const int64_t off = ((tok_base + t0 + t) * a.Hv + h) * DK * gsz + p * 16;
      cp_async16(raw + Tr::kRawG + t * DK * gsz + p * 16, g + off);
    }
    constexpr int vp = kBV * 2 / 16;
    for (int i = tid; i < n * vp; i += kThreads) {
      const int t = i / vp, p = i % vp;
      const int64_t off = ((tok_base + t0 + t) * a.Hv + h) * a.dv + col0 + p * 8;
      cp_async16(raw + Tr::kRawV + (t * kBV + p * 8) * 2, v + off);
    }
    if (tid < n) {
      // the aligned 32-bit word holding this token's beta (beta is 4-byte aligned)
      const uintptr_t e =
          reinterpret_cast<uintptr_t>(beta + ((tok_base + t0 + tid) * a.Hv + h) * bsz);
      cp_async4(raw + Tr::kRawBeta + tid * 4, reinterpret_cast<const void*>(e & ~uintptr_t(3)));
    }
    cp_async_commit();
  };

  auto convert = [&](int c) {
    const unsigned char* raw = smem + (c & 1) * Tr::kRawBytes;
    const int t0 = c * kTC, n = min(kTC, T - t0);
    constexpr int qp = DK / 8;
    for (int i = tid; i < n * qp; i += kThreads) {
      const int t = i / qp, r = (i % qp) * 8;
      const int dst = t * Tr::kVec + (r / Tr::kRows) * Tr::kPad + (r % Tr::kRows);
      float f[8];
      unpack8<IO>(*reinterpret_cast<const uint4*>(raw + Tr::kRawQ + (t * DK + r) * 2), f);
      *reinterpret_cast<float4*>(sQ + dst) =
          make_float4(f[0] * a.scale, f[1] * a.scale, f[2] * a.scale, f[3] * a.scale);
      *reinterpret_cast<float4*>(sQ + dst + 4) =
          make_float4(f[4] * a.scale, f[5] * a.scale, f[6] * a.scale, f[7] * a.scale);
      unpack8<IO>(*reinterpret_cast<const uint4*>(raw + Tr::kRawK + (t * DK + r) * 2), f);
      *reinterpret_cast<float4*>(sK + dst) = make_float4(f[0], f[1], f[2], f[3]);
      *reinterpret_cast<float4*>(sK + dst + 4) = make_float4(f[4], f[5], f[6], f[7]);
    }
    for (int i = tid; i < n * (DK / 4); i += kThreads) {
      const int t = i / (DK / 4), r = (i % (DK / 4)) * 4;
      const unsigned char* row = raw + Tr::kRawG + t * DK * gsz;
      const int dst = t * Tr::kVec + (r / Tr::kRows) * Tr::kPad + (r % Tr::kRows);
      *reinterpret_cast<float4*>(sE + dst) =
          make_float4(expf(smem_any(row, r, a.g_dtype)), expf(smem_any(row, r + 1, a.g_dtype)),
                      expf(smem_any(row, r + 2, a.g_dtype)), expf(smem_any(row, r + 3, a.g_dtype)));
    }
    for (int i = tid; i < n * (kBV / 8); i += kThreads) {
      const int t = i / (kBV / 8), cc = (i % (kBV / 8)) * 8;
      float f[8];
      unpack8<IO>(*reinterpret_cast<const uint4*>(raw + Tr::kRawV + (t * kBV + cc) * 2), f);
      *reinterpret_cast<float4*>(sV + t * kBV + cc) = make_float4(f[0], f[1], f[2], f[3]);
      *reinterpret_cast<float4*>(sV + t * kBV + cc + 4) = make_float4(f[4], f[5], f[6], f[7]);
    }
    if (tid < n) {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(raw + Tr::kRawBeta + tid * 4);
      float bt;
      if (a.beta_dtype == GDN_DT_F32) {
        bt = __uint_as_float(w);
      } else {
        const uintptr_t e =
            reinterpret_cast<uintptr_t>(beta + ((tok_base + t0 + tid) * a.Hv + h) * bsz);
        const unsigned short r16 = static_cast<unsigned short>((e & 2) ? (w >> 16) : (w & 0xFFFFu));
        bt = a.beta_dtype == GDN_DT_BF16 ? __uint_as_float(static_cast<uint32_t>(r16) << 16)
                                         : __half2float(__ushort_as_half(r16));
      }
      sBeta[tid] = bt;
    }
    for (int t = warp; t < n; t += kThreads / 32) {
      const IO* rq = reinterpret_cast<const IO*>(raw + Tr::kRawQ) + t * DK;
      const IO* rk = reinterpret_cast<const IO*>(raw + Tr::kRawK) + t * DK;
      float d = 0.f;
#pragma unroll
      for (int j = lane; j < DK; j += 32) d = fmaf(to_f32<IO>(rq[j]), to_f32<IO>(rk[j]), d);
#pragma unroll
      for (int m = 16; m; m >>= 1) d += __shfl_xor_sync(0xffffffffu, d, m);
      if (lane == 0) sQK[t] = d * a.scale;
    }
  };

  auto flush = [&](int c) {
    const int t0 = c * kTC, n = min(kTC, T - t0);
    constexpr int op = kBV * 2 / 16;
    for (int i = tid; i < n * op; i += kThreads) {
      const int t = i / op, p = i % op;
      const int64_t off = ((tok_base + t0 + t) * a.Hv + h) * a.dv + col0 + p * 8;
      *reinterpret_cast<uint4*>(o + off) = *reinterpret_cast<const uint4*>(sO + t * kBV + p * 8);
    }
  };

  // state column `col0 + col`, rows qt*kRows .. qt*kRows + kRows - 1
  float s[Tr::kRows];
  const int64_t srow0 = (static_cast<int64_t>(bh) * DK + qt * Tr::kRows) * a.dv + col0 + col;
  if (a.initial_state) {
    const float* S0 = a.initial_state;
#pragma unroll
    for (int i = 0; i < Tr::kRows; ++i) s[i] = __ldg(S0 + srow0 + static_cast<int64_t>(i) * a.dv);
  } else {
#pragma unroll
    for (int i = 0; i < Tr::kRows; ++i) s[i] = 0.f;
  }

  issue(0);
  for (int c = 0; c < nchunks; ++c) {
    cp_async_wait_all();
    __syncthreads();  // chunk c staged; chunk c-1's compute is done
    if (c + 1 < nchunks) issue(c + 1);
    if (c > 0) flush(c - 1);
    convert(c);
    __syncthreads();
    const int n = min(kTC, T - c * kTC);
    const float* eb = sE + qt * Tr::kPad;
    const float* kb = sK + qt * Tr::kPad;
    const float* qb = sQ + qt * Tr::kPad;
    for (int t = 0; t < n; ++t) {
      const float* et = eb + t * Tr::kVec;
      const float* kt = kb + t * Tr::kVec;
      const float* qtv = qb + t * Tr::kVec;
      float u0 = 0.f, u1 = 0.f, u2 = 0.f, u3 = 0.f, p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
#pragma unroll
      for (int i = 0; i < Tr::kRows; i += 4) {
        const float4 e4 = lds128(et + i), k4 = lds128(kt + i), q4 = lds128(qtv + i);
        s[i] *= e4.x;
        s[i + 1] *= e4.y;
        s[i + 2] *= e4.z;
        s[i + 3] *= e4.w;
        u0 = fmaf(k4.x, s[i], u0);
        u1 = fmaf(k4.y, s[i + 1], u1);
        u2 = fmaf(k4.z, s[i + 2], u2);
        u3 = fmaf(k4.w, s[i + 3], u3);
        p0 = fmaf(q4.x, s[i], p0);
        p1 = fmaf(q4.y, s[i + 1], p1);
        p2 = fmaf(q4.z, s[i + 2], p2);
        p3 = fmaf(q4.w, s[i + 3], p3);
      }
      float u = (u0 + u1) + (u2 + u3), p = (p0 + p1) + (p2 + p3);
      u += __shfl_xor_sync(0xffffffffu, u, 8);
      p += __shfl_xor_sync(0xffffffffu, p, 8);
      u += __shfl_xor_sync(0xffffffffu, u, 16);
      p += __shfl_xor_sync(0xffffffffu, p, 16);
      const float br = sBeta[t] * (sV[t * kBV + col] - u);
      if (qt == 0) sO[t * kBV + col] = from_f32<IO>(fmaf(sQK[t], br, p));
#pragma unroll
      for (int i = 0; i < Tr::kRows; i += 4) {
        const float4 k4 = lds128(kt + i);
        s[i] = fmaf(k4.x, br, s[i]);
        s[i + 1] = fmaf(k4.y, br, s[i + 1]);
        s[i + 2] = fmaf(k4.z, br, s[i + 2]);
        s[i + 3] = fmaf(k4.w, br, s[i + 3]);
      }
    }
  }
  __syncthreads();
  flush(nchunks - 1);
  float* S1 = a.final_state;
#pragma unroll
  for (int i = 0; i < Tr::kRows; ++i) S1[srow0 + static_cast<int64_t>(i) * a.dv] = s[i];
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

extern "C" int kda_prefill_launch(const gdn_prefill_args_t* args, gdn_stream_t stream) {
  int rc = gdn::kda_prefill::validate(args);
  if (rc) return rc;
  gdn::DeviceInfo di;
  if ((rc = gdn::device_info(&di))) return rc;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  return args->io_dtype == GDN_DT_BF16 ? gdn::kda_prefill::launch<__nv_bfloat16>(*args, s)
                                       : gdn::kda_prefill::launch<__half>(*args, s);
}
