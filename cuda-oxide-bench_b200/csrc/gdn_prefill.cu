// gdn_prefill.cu — GDN chunked prefill on the sm_100a tensor cores (tcgen05).
//
// The reference defines prefill only as T applications of its decode
// recurrence (pytorch_reference_gdn.py:38-91; chunking is described, not
// implemented, in analysis/wave15-attention-research/MECHANISMS.md:398-445).
// This code computes the same result chunk by chunk (chunk C = 64 tokens).
// Per chunk, with G the in-chunk cumulative log gate, gamma = exp(G):
//   A[i][j] = beta_i exp(G_i - G_j) k_i.k_j            (j < i)
//   T       = (I + A)^-1                                (blocked forward substitution, fp32)
//   W       = T diag(beta gamma) K,   U = T diag(beta) V
//   V'      = U - W S                                   (S: state entering the chunk)
//   O       = diag(gamma) Q S + (Q K^T . causal . exp(G_i - G_j)) V'
//   S_next  = gamma_C S + K^T diag(exp(G_C - G_j)) V'
// which unrolls the recurrence S_t = a_t S_{t-1} + beta_t k_t (v_t - a_t S_{t-1}^T k_t)^T
// exactly (in exact arithmetic).
//
// Two kernels.  Everything that does not depend on the state (the gated
// K K^T / Q K^T products, the solve, T_w = T diag(beta gamma), T_u = T diag(beta)
// and the causal decayed P = Q K^T . causal . exp(G_i - G_j)) is independent
// across chunks, so the first kernel (intra_kernel) computes it for every
// (batch, q/k head, chunk) at once — 4096 CTAs at config 3, three per SM — and
// writes bf16 T_w, T_u, P tiles (already in the 128B-swizzled shared-memory
// layout) plus the fp32 gamma / decay vectors to a workspace.  The second
// kernel (state_kernel, one CTA per (batch, value head)) runs only the serial
// state chain over the chunks, fed from the workspace by bulk copies:
//   helper warps 0-7:  W^T = K^T T_w^T and U^T = V^T T_u^T (tcgen05), the bf16
//                      W^T tile, outputs of the previous chunk, refills;
//   state warps 8-15:  V'^T = U^T - S^T W^T (S^T from TMEM, negated A), the
//                      V'^T / V''^T hi / lo tiles, dS^T = V''^T K (hi + lo),
//                      Z^T = S^T Q^T, O_intra^T = V'^T P^T, the fp32 state
//                      update in registers and the bf16 S^T written back to TMEM.
// Every product is a tcgen05.mma with M = 128, written transposed so the 128
// TMEM lanes index d_v (or d_k).  Operands are bf16 (f16) in 128B-swizzled
// shared memory; S^T lives in TMEM as bf16 and is read as the A operand.
// Precision: the decayed V'' = diag(exp(G_C - G_j)) V' that updates the state
// is split into bf16 hi + lo halves (two MMAs), and K enters the state update
// unscaled, so the state accumulates with ~16 mantissa bits per term.
// Hand-offs use mbarriers (TMA / bulk-copy bytes, tcgen05.commit, group
// arrivals); every wait is bounded and each group agrees on an abort before
// leaving its loop.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "ptx.cuh"
#include "tc.cuh"

namespace gdn {
namespace prefill {

constexpr int kC = 64;     // chunk length
constexpr int kD = 128;    // d_k = d_v
constexpr int kLd = 68;    // fp32 row stride of the solver matrices

#ifdef GDN_PREFILL_TRACE
// Phase timestamps of CTA 0 of the state kernel (profiling builds only): [chunk][phase].
__device__ unsigned long long g_trace[64 * 16];
#define TRACE(c, ph)                                                                           \
  do {                                                                                         \
    if (blockIdx.x == 0 && (c) < 64 && (threadIdx.x & 127) == 0 && threadIdx.x < 384)        \
      g_trace[(c) * 16 + (ph)] = clock64();                                                    \
  } while (0)
__device__ unsigned long long g_trace1[4096 * 8];
__device__ unsigned long long g_cta[8192 * 5];  // start, end (globaltimer), smid, setup done, compute done
#define TRACE1(ph)                                                                       \
  do {                                                                                   \
    if (blockIdx.x < 4096 && threadIdx.x == 0) g_trace1[blockIdx.x * 8 + (ph)] = global_timer_ns(); \
  } while (0)
// per-CTA phase clocks of the KDA intra kernel (SM cycles)
__device__ unsigned long long g_ktrace[4096 * 16];
#define KTRACE(ph)                                                                          \
  do {                                                                                      \
    if (blockIdx.x < 4096 && threadIdx.x == 0) g_ktrace[blockIdx.x * 16 + (ph)] = clock64(); \
  } while (0)
#else
#define KTRACE(ph) \
  do {             \
  } while (0)
#define TRACE1(ph) \
  do {             \
  } while (0)
#define TRACE(c, ph) \
  do {               \
  } while (0)
#endif

// Workspace record of one (batch, value head, chunk): bf16 tiles in the
// 128B-swizzled layout of a 64 x 64 K-major operand (rows i, 1024-byte
// atoms), then the fp32 vectors.
constexpr uint32_t kWsTw = 0;        // T diag(beta gamma)   rows i, cols j
constexpr uint32_t kWsTu = 8192;     // T diag(beta)
constexpr uint32_t kWsP = 16384;     // Q K^T . causal . exp(G_i - G_j)
constexpr uint32_t kWsVec = 24576;   // gamma[64], exp(G_C - G_j)[64] fp32
constexpr uint32_t kWsUnit = 25088;
static_assert(kWsUnit % 16 == 0 && kWsP % 16 == 0 && kWsVec % 16 == 0, "bulk-copy alignment");

// Workspace record of the KDA (per-channel gate) prefill, one per (batch,
// value head, chunk).  The per-channel decays cannot be applied as row
// scales inside the state pass, so the intra kernel hands over operands that
// already carry them (G: in-chunk cumulative log gate, per token and channel):
constexpr uint32_t kKWsTu = 0;       // T diag(beta), K-major rows i             (8 KB)
constexpr uint32_t kKWsP = 8192;     // (Q K^T)_ij over channels with exp(G_i - G_j), causal (8 KB)
constexpr uint32_t kKWsWT = 16384;   // W^T = (T diag(beta) (K . exp(G)))^T, MN-major rows d_k (16 KB)
constexpr uint32_t kKWsQT = 32768;   // (Q . exp(G))^T, MN-major rows d_k          (16 KB)
constexpr uint32_t kKWsKd = 49152;   // K . exp(G_C - G) as f16, the K tile layout (16 KB)
constexpr uint32_t kKWsVec = 65536;  // exp(G_C)[d_k] fp32                         (512 B)
constexpr uint32_t kKWsUnit = 66048;
static_assert(kKWsUnit % 16 == 0, "bulk-copy alignment");

struct Params {
  gdn_prefill_args_t a;
  int32_t nchunks;
  int32_t group;
  unsigned char* ws;
  uint32_t* slow_count;  // KDA: units deferred to the slow-path kernel, and their list
  int32_t* slow_list;
};

template <bool BF16>
__device__ __forceinline__ void store_row16(uint32_t tile, int row, int chunk0, const float* v) {
  tc::sts128(tile + tc::sw128_offset(row, chunk0), tc::pack2<BF16>(v[0], v[1]),
             tc::pack2<BF16>(v[2], v[3]), tc::pack2<BF16>(v[4], v[5]), tc::pack2<BF16>(v[6], v[7]));
  tc::sts128(tile + tc::sw128_offset(row, chunk0 + 1), tc::pack2<BF16>(v[8], v[9]),
             tc::pack2<BF16>(v[10], v[11]), tc::pack2<BF16>(v[12], v[13]),
             tc::pack2<BF16>(v[14], v[15]));
}

// Same layout, written to a global-memory copy of the tile.
template <bool BF16>
__device__ __forceinline__ void store_row16_global(unsigned char* tile, int row, int chunk0,
                                                   const float* v) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const float* w = v + 8 * h;
    uint4 u = make_uint4(tc::pack2<BF16>(w[0], w[1]), tc::pack2<BF16>(w[2], w[3]),
                         tc::pack2<BF16>(w[4], w[5]), tc::pack2<BF16>(w[6], w[7]));
    *reinterpret_cast<uint4*>(tile + tc::sw128_offset(row, chunk0 + h)) = u;
  }
}

// Bounded wait polled by lane 0 of each warp (the other lanes sleep in the
// barrier instead of competing for issue slots), then a group-wide vote: the
// group leaves together if any warp timed out (no thread is stranded at a
// barrier).  The barrier also orders the waiters' later reads after the phase.
__device__ __forceinline__ bool group_wait(uint64_t* bar, uint32_t parity, int bar_id, int count,
                                           bool failed = false) {
  bool ok = !failed;
  if ((threadIdx.x & 31) == 0 && ok) ok = mbar_wait_bounded(bar, parity);
  return !named_barrier_or(bar_id, count, !ok);
}

// ------------------------------------------------------------ triangular solve
// m16n8k8 TF32 warp MMA for the block products of the solve.  A single TF32
// product (10-bit mantissa, ~5e-4 relative) is enough: T is rounded to bf16
// (~4e-3 relative) right after the solve, before any use.  The tensor core
// reads only the tf32 bits of its fp32 operands.
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

constexpr int kMsLd = 36;  // fp32 row stride of the solver scratch (32 columns + 4)

// acc (16 x 16, two m16n8 fragments) += X (16 x 16 block at x, row stride
// LX) * Y (16 x 16 at y, row stride LY).
template <int LX = kLd, int LY = kLd>
__device__ __forceinline__ void block_mma(float (&acc)[2][4], const float* x, const float* y, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int ks = 0; ks < 2; ++ks) {
    uint32_t af[4];
    af[0] = __float_as_uint(x[g * LX + ks * 8 + t]);
    af[1] = __float_as_uint(x[(g + 8) * LX + ks * 8 + t]);
    af[2] = __float_as_uint(x[g * LX + ks * 8 + t + 4]);
    af[3] = __float_as_uint(x[(g + 8) * LX + ks * 8 + t + 4]);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      uint32_t bf[2];
      bf[0] = __float_as_uint(y[(ks * 8 + t) * LY + nt * 8 + g]);
      bf[1] = __float_as_uint(y[(ks * 8 + t + 4) * LY + nt * 8 + g]);
      mma_tf32(acc[nt], af, bf);
    }
  }
}

template <int LZ = kLd>
__device__ __forceinline__ void block_store(float* z, const float (&acc)[2][4], float sign, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    *reinterpret_cast<float2*>(z + g * LZ + nt * 8 + 2 * t) = make_float2(sign * acc[nt][0], sign * acc[nt][1]);
    *reinterpret_cast<float2*>(z + (g + 8) * LZ + nt * 8 + 2 * t) =
        make_float2(sign * acc[nt][2], sign * acc[nt][3]);
  }
}

// In place: AT holds strictly-lower A (64 x 64 fp32, stride kLd, zeros on and
// above the diagonal) and is overwritten with T = (I + A)^-1.  Run by one
// group of four warps (w = 0..3 inside the group) that syncs on named barrier
// `bar` (128 threads).  Steps: the four 16 x 16 diagonal blocks D_r by forward
// substitution (one warp each, one lane per column, fp32); T_10 = -D_1 A_10 D_0
// and T_32 = -D_3 A_32 D_2; then the lower-left quadrant -T_bot A_bl T_top
// through Y = A_bl T_top (TF32 warp MMAs).  Each block of A is last read
// before the block of T that replaces it is written.  M is [32][kMsLd] scratch.
__device__ __forceinline__ void solve_unit_lower(float* AT, float* M, int w, int lane, int bar) {
  {
    const int bb = w * 16, c = lane & 15;
    float t[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) t[i] = (i == c) ? 1.f : 0.f;
#pragma unroll
    for (int i = 1; i < 16; ++i) {
      const float* row = AT + (bb + i) * kLd + bb;
      // four partial sums (j mod 4) shorten the dependent FMA chain
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j4 = 0; j4 < i; j4 += 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(row + j4);
        acc[0] = fmaf(a4.x, t[j4], acc[0]);
        if (j4 + 1 < i) acc[1] = fmaf(a4.y, t[j4 + 1], acc[1]);
        if (j4 + 2 < i) acc[2] = fmaf(a4.z, t[j4 + 2], acc[2]);
        if (j4 + 3 < i) acc[3] = fmaf(a4.w, t[j4 + 3], acc[3]);
      }
      t[i] -= (acc[0] + acc[1]) + (acc[2] + acc[3]);
    }
    __syncwarp();
    if (lane < 16) {
#pragma unroll
      for (int i = 0; i < 16; ++i) AT[(bb + i) * kLd + bb + c] = t[i];
    }
  }
  tc::group_sync(bar, 128);
  if (w < 2) {  // T_10 (w 0) and T_32 (w 1)
    const int c = w * 2, r = c + 1;
    float* X = M + w * 16 * kMsLd;
    float acc[2][4] = {};
    block_mma(acc, AT + 16 * r * kLd + 16 * c, AT + 16 * c * kLd + 16 * c, lane);
    block_store<kMsLd>(X, acc, 1.f, lane);
    __syncwarp();
    float acc2[2][4] = {};
    block_mma<kLd, kMsLd>(acc2, AT + 16 * r * kLd + 16 * r, X, lane);
    block_store(AT + 16 * r * kLd + 16 * c, acc2, -1.f, lane);
  }
  tc::group_sync(bar, 128);
  {  // Y_rc = sum_k A_rk T_kc over the top blocks, warp (r-2)*2 + c
    const int r = 2 + (w >> 1), c = w & 1;
    float acc[2][4] = {};
    if (c == 0) {
      block_mma(acc, AT + 16 * r * kLd + 0, AT + 0, lane);                      // A_r0 D_0
      block_mma(acc, AT + 16 * r * kLd + 16, AT + 16 * kLd + 0, lane);          // A_r1 T_10
    } else {
      block_mma(acc, AT + 16 * r * kLd + 16, AT + 16 * kLd + 16, lane);         // A_r1 D_1
    }
    block_store<kMsLd>(M + (r - 2) * 16 * kMsLd + 16 * c, acc, 1.f, lane);
  }
  tc::group_sync(bar, 128);
  {
    const int r = 2 + (w >> 1), c = w & 1;
    float acc[2][4] = {};
    if (r == 2) {
      block_mma<kLd, kMsLd>(acc, AT + 32 * kLd + 32, M + 16 * c, lane);         // D_2 Y_2c
    } else {
      block_mma<kLd, kMsLd>(acc, AT + 48 * kLd + 32, M + 16 * c, lane);         // T_32 Y_2c
      block_mma<kLd, kMsLd>(acc, AT + 48 * kLd + 48, M + 16 * kMsLd + 16 * c, lane);  // D_3 Y_3c
    }
    block_store(AT + 16 * r * kLd + 16 * c, acc, -1.f, lane);
  }
  tc::group_sync(bar, 128);
}

// ============================================================ intra kernel
// One CTA per (batch, q/k head, chunk), 8 warps; warps 4h..4h+3 serve value
// head (pair index) h of the q/k head's group, so a GQA pair shares the
// K K^T / Q K^T product.  Chunks run last-to-first so that the state kernel,
// which starts at chunk 0, finds the most recent records still in L2.
#ifndef GDN_K1_MINB
#define GDN_K1_MINB 3
#endif
namespace intra {
constexpr int kThreads = 256;
constexpr uint32_t kKQ = 0;                      // [K | Q] per d_k block: 2 x 16 KB
constexpr uint32_t kKQBlock = 16384;
constexpr uint32_t kATHead = 64 * kLd * 4;       // 17408
constexpr uint32_t kAT = 32768;                  // [2 heads] A -> T in place
constexpr uint32_t kMsHead = 32 * kMsLd * 4;     // 4608: solver scratch per head, aliasing
                                                 // the K/Q tiles once the MMA is done
constexpr uint32_t kPStage = 2 * kMsHead;        // [2 heads] P tile (8 KB), likewise
constexpr uint32_t kVec = kAT + 2 * kATHead;     // [2 heads][G|beta|gamma|decay|Ee|Es][64]
constexpr uint32_t kFlags = kVec + 2 * 6 * 64 * 4;
constexpr uint32_t kBars = kFlags + 16;
constexpr uint32_t kSmemBytes = kBars + 64;
constexpr uint32_t kSmemAlloc = kSmemBytes + 1024;
static_assert(kPStage + 2 * 8192 <= kAT, "solver scratch and P tiles overflow the K/Q tiles");
}  // namespace intra

template <bool BF16>
__global__ void __launch_bounds__(intra::kThreads, GDN_K1_MINB)
    intra_kernel(const Params p, const __grid_constant__ CUtensorMap map_q,
                 const __grid_constant__ CUtensorMap map_k) {
  using namespace intra;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBars);  // [0] TMA, [1] MMA
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2);

#ifdef GDN_PREFILL_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 8192) {
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    g_cta[blockIdx.x * 5] = global_timer_ns();
    g_cta[blockIdx.x * 5 + 2] = smid;
  }
#endif
  const gdn_prefill_args_t& a = p.a;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hh = warp >> 2, w4 = warp & 3, ht = tid & 127;
  const int per_c = a.B * a.Hqk;
  const int c = p.nchunks - 1 - static_cast<int>(blockIdx.x) / per_c;
  const int bq = static_cast<int>(blockIdx.x) % per_c;
  const int b = bq / a.Hqk, hq = bq % a.Hqk;
  const int T = a.T, t0 = c * kC;

  // raw gate and beta of token ht of value head (pair slot) hh, pair p0;
  // issued before anything else so that their latency overlaps the set-up
  // (as raw bits: the conversion, and with it the wait for the load, happens
  // at first use)
  auto load_raw = [](const void* base, int64_t i, int dt) -> uint32_t {
    if (dt == GDN_DT_F32) return __ldg(reinterpret_cast<const uint32_t*>(base) + i);
    return __ldg(reinterpret_cast<const unsigned short*>(base) + i);
  };
  auto from_raw = [](uint32_t raw, int dt) -> float {
    if (dt == GDN_DT_F32) return __uint_as_float(raw);
    if (dt == GDN_DT_BF16) return __uint_as_float(raw << 16);
    return __half2float(__ushort_as_half(static_cast<unsigned short>(raw)));
  };
  auto load_gate = [&](int p0, uint32_t& gv, uint32_t& bv) {
    gv = 0u;  // padded tokens: no decay, no update (0 in every dtype)
    bv = 0u;
    const int t = t0 + ht;
    if (p0 + hh < p.group && ht < kC && t < T) {
      const int64_t gi = (static_cast<int64_t>(b) * T + t) * a.Hv + hq * p.group + p0 + hh;
      gv = load_raw(a.g, gi, a.g_dtype);
      bv = load_raw(a.beta, gi, a.beta_dtype);
    }
  };
  // With programmatic dependent launch this kernel may start while the
  // previous kernel in the stream drains: wait for it before the first
  // global read, then let the state-pass kernel start its own prologue.
  pdl_wait();
  pdl_launch_dependents();
  uint32_t gv0, bv0;
  load_gate(0, gv0, bv0);
  if (warp == 0) tc::tmem_alloc(tmem_holder, 64);
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  const uint32_t lane_base = static_cast<uint32_t>(w4 * 32) << 16;
  constexpr uint32_t kIdKQ = tc::idesc_f16(128, 64, false, false, BF16);

  const int bar = 2 + hh;
  float* AT = reinterpret_cast<float*>(smem + kAT + hh * kATHead);
  float* Ms = reinterpret_cast<float*>(smem + kKQ + hh * kMsHead);
  float* sG = reinterpret_cast<float*>(smem + kVec) + hh * 384;
  float* sBeta = sG + 64;
  float* sGam = sG + 128;
  float* sDec = sG + 192;
  float* sEe = sG + 256;   // exp(G_end(J) - G_j)
  float* sEs = sG + 320;   // exp(G_start(J) - G_j)
  int* sFast = reinterpret_cast<int*>(smem + kFlags) + hh;
  // The in-chunk cumulative log gate of value head (pair slot) hh of pair p0
  // and the exponentials derived from it (independent of the K/Q tiles).
  auto gates = [&](int p0, uint32_t graw, uint32_t braw) {
    const bool active = p0 + hh < p.group;
    const int h = hq * p.group + p0 + hh;
    unsigned char* rec = p.ws + (static_cast<size_t>(b * a.Hv + h) * p.nchunks + c) * kWsUnit;
    if (active && ht < kC) {
      sG[ht] = from_raw(graw, a.g_dtype);
      sBeta[ht] = from_raw(braw, a.beta_dtype);
    }
    tc::group_sync(bar, 128);
    if (active && w4 == 0) {  // in-chunk cumulative log gate; lane l owns tokens 2l, 2l+1
      const float g0 = sG[2 * lane], g1 = sG[2 * lane + 1];
      float run = g0 + g1;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float o = __shfl_up_sync(0xffffffffu, run, off);
        if (lane >= off) run += o;
      }
      const float excl = run - (g0 + g1);
      const float GC = __shfl_sync(0xffffffffu, run, 31);
      const float Ga = excl + g0, Gb = run;
      // G at the first and last token of this lane's 16-token block
      const float Gs = __shfl_sync(0xffffffffu, Ga, lane & ~7);
      const float Ge = __shfl_sync(0xffffffffu, Gb, lane | 7);
      // the factored exponentials below stay finite when no block decays by
      // more than 80 (nats) within itself; otherwise the direct form is used
      const bool fast = __all_sync(0xffffffffu, Gs - Ge <= 80.f);
      __syncwarp();
      sG[2 * lane] = Ga;
      sG[2 * lane + 1] = Gb;
      const float2 gam = make_float2(__expf(Ga), __expf(Gb));
      const float2 dec = make_float2(__expf(GC - Ga), __expf(GC - Gb));  // V'' row scale
      reinterpret_cast<float2*>(sGam)[lane] = gam;
      reinterpret_cast<float2*>(sDec)[lane] = dec;
      reinterpret_cast<float2*>(sEe)[lane] = make_float2(__expf(Ge - Ga), __expf(Ge - Gb));
      reinterpret_cast<float2*>(sEs)[lane] =
          make_float2(__expf(fminf(Gs - Ga, 80.f)), __expf(fminf(Gs - Gb, 80.f)));
      if (lane == 0) *sFast = fast ? 1 : 0;
      reinterpret_cast<float2*>(rec + kWsVec)[lane] = gam;
      reinterpret_cast<float2*>(rec + kWsVec + 256)[lane] = dec;
    }
    tc::group_sync(bar, 128);
  };
  TRACE1(0);
#ifdef GDN_PREFILL_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 8192) g_cta[blockIdx.x * 5 + 3] = global_timer_ns();
#endif
  if (tid == 0) {
    mbar_arrive_expect_tx(&bars[0], 4 * 8192);
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
    unsigned char* kq = smem + kKQ + blk * kKQBlock;
    tc::tma_load_4d(kq, &map_k, blk * 64, hq, t0, b, &bars[0]);
    tc::tma_load_4d(kq + 8192, &map_q, blk * 64, hq, t0, b, &bars[0]);
    }
  }
  gates(0, gv0, bv0);  // while the K/Q tiles are in flight
  bool ok = true;
  if (tid == 0) {
    // [K;Q] K^T: TMEM lanes 0-63 hold K K^T rows, lanes 64-127 Q K^T rows
    ok = mbar_wait_bounded(&bars[0], 0);
    if (ok) {
      tc::fence_after_sync();
#pragma unroll
      for (int s = 0; s < 8; ++s)
        tc::mma(tmem, tc::kmajor_desc(sb + kKQ, kKQBlock, s), tc::kmajor_desc(sb + kKQ, kKQBlock, s),
                kIdKQ, s > 0);
      tc::commit(&bars[1]);
    }
  }
  // Every warp learns whether the product is coming; lane 0 of each warp then
  // waits for it (bounded) and the CTA votes.
  ok = !named_barrier_or(1, kThreads, !ok);
  if (ok) {
    bool mine = true;
    if (lane == 0) mine = mbar_wait_bounded(&bars[1], 0);
    ok = !named_barrier_or(1, kThreads, !mine);
  }
  TRACE1(1);
  if (!ok) {
    if (tid == 0) report(a.status, GDN_DEVERR_MMA_TIMEOUT);
  } else {
    tc::fence_after_sync();
    for (int p0 = 0; p0 < p.group; p0 += 2) {
      const bool active = p0 + hh < p.group;  // an odd group leaves warps 4-7 idle
      const int h = hq * p.group + p0 + hh;
      unsigned char* rec = p.ws + (static_cast<size_t>(b * a.Hv + h) * p.nchunks + c) * kWsUnit;
      if (p0 > 0) {
        if (ht == 64) bulk_wait_read();  // the previous pair's P tile has left
        uint32_t gv, bv;
        load_gate(p0, gv, bv);
        gates(p0, gv, bv);
      }
      TRACE1(2);
      if (active) {  // A rows (TMEM lanes 0-63, warps 0-1) and P rows (lanes 64-127, warps 2-3)
        // exp(G_i - G_j) for j <= i, factored by 16-token blocks I = i/16, J = j/16:
        //   J < I : exp(G_i - G_end(J)) exp(G_end(J) - G_j)     (both factors <= 1)
        //   J = I : exp(G_i - G_start(I)) exp(G_start(I) - G_j) (fast path) or direct
        // so each row needs four exponentials instead of one per element.
        const int i = (w4 & 1) * 32 + lane;
        const int I = i >> 4;
        const float Gi = sG[i];
        const float bi = sBeta[i];
        const bool fast = *sFast != 0;
        float rf[3];
#pragma unroll
        for (int J = 0; J < 3; ++J) rf[J] = (J < I) ? __expf(Gi - sG[16 * J + 15]) : 0.f;
        const float rd = __expf(Gi - sG[16 * I]);
#pragma unroll
        for (int cb = 0; cb < 2; ++cb) {
          float r[32];
          if ((w4 & 1) == 0 && cb == 1) {  // rows 0-31, columns 32-63: above the diagonal
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) r[jj] = 0.f;
          } else {
            tc::tmem_ld16(tmem + lane_base + cb * 32, *reinterpret_cast<float(*)[16]>(r));
            tc::tmem_ld16(tmem + lane_base + cb * 32 + 16, *reinterpret_cast<float(*)[16]>(r + 16));
            tc::tmem_wait_ld();
            const float row_s = w4 < 2 ? bi : 1.f;
            const int lim = w4 < 2 ? i : i + 1;  // A: j < i; P: j <= i
            if (fast) {
              // per 16-column block J: the warp's rows lie in blocks Ia and
              // Ia + 1, so blocks below Ia need no mask and one product per
              // element, blocks above Ia + 1 are zero, and only the two
              // blocks at Ia, Ia + 1 take the general form
              const int Ia = 2 * (w4 & 1);
#pragma unroll
              for (int jb = 0; jb < 2; ++jb) {
                const int J = 2 * cb + jb;
                float* rb = r + 16 * jb;
                if (J < Ia) {
                  const float f = row_s * rf[J < 3 ? J : 2];
#pragma unroll
                  for (int e4 = 0; e4 < 16; e4 += 4) {
                    const float4 ee = *reinterpret_cast<const float4*>(sEe + 16 * J + e4);
                    rb[e4] *= f * ee.x; rb[e4 + 1] *= f * ee.y; rb[e4 + 2] *= f * ee.z; rb[e4 + 3] *= f * ee.w;
                  }
                } else if (J > Ia + 1) {
#pragma unroll
                  for (int jj = 0; jj < 16; ++jj) rb[jj] = 0.f;
                } else {
                  const float fo = row_s * rf[J < 3 ? J : 2], fd = row_s * rd;
#pragma unroll
                  for (int e4 = 0; e4 < 16; e4 += 4) {
                    const float4 ee = *reinterpret_cast<const float4*>(sEe + 16 * J + e4);
                    const float4 es = *reinterpret_cast<const float4*>(sEs + 16 * J + e4);
                    const float eo[4] = {ee.x, ee.y, ee.z, ee.w}, ed[4] = {es.x, es.y, es.z, es.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                      const int j = 16 * J + e4 + q;
                      const float e = (J < I) ? fo * eo[q] : fd * ed[q];
                      rb[e4 + q] = (j < lim) ? e * rb[e4 + q] : 0.f;
                    }
                  }
                }
              }
            } else {
#pragma unroll
              for (int jj = 0; jj < 32; ++jj) {
                const int j = cb * 32 + jj;
                r[jj] = (j < lim) ? row_s * __expf(Gi - sG[j]) * r[jj] : 0.f;
              }
            }
          }
          if (w4 < 2) {
#pragma unroll
            for (int j4 = 0; j4 < 32; j4 += 4)
              *reinterpret_cast<float4*>(AT + i * kLd + cb * 32 + j4) =
                  make_float4(r[j4], r[j4 + 1], r[j4 + 2], r[j4 + 3]);
          } else {
            const uint32_t pst = sb + kKQ + kPStage + hh * 8192;
            store_row16<BF16>(pst, i, cb * 4, r);
            store_row16<BF16>(pst, i, cb * 4 + 2, r + 16);
          }
        }
        if (w4 >= 2) tc::fence_proxy_async();  // the P tile is read by a bulk copy
      }
      tc::group_sync(bar, 128);
      if (active && ht == 64) {  // the whole P tile to its record in one bulk copy
        bulk_s2g(rec + kWsP, smem + kKQ + kPStage + hh * 8192, 8192);
        bulk_commit();
      }
      TRACE1(3);
      if (active) solve_unit_lower(AT, Ms, w4, lane, bar);
      TRACE1(4);
      if (active) {
        // T_w = T diag(beta gamma), T_u = T diag(beta).  Warp w4 writes rows
        // 16 w4 .. 16 w4 + 15; lane l the 16-byte chunk l % 8 (columns
        // 8 (l % 8) ..) of rows 16 w4 + l / 8 + 4 s, so each store instruction
        // covers four whole 128-byte rows (512 contiguous bytes).
        const int ch = lane & 7;
        const float4 b0 = *reinterpret_cast<const float4*>(sBeta + 8 * ch);
        const float4 b1 = *reinterpret_cast<const float4*>(sBeta + 8 * ch + 4);
        const float4 g0 = *reinterpret_cast<const float4*>(sGam + 8 * ch);
        const float4 g1 = *reinterpret_cast<const float4*>(sGam + 8 * ch + 4);
        const float bj[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        const float gj[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
        for (int s4 = 0; s4 < 4; ++s4) {
          const int i = 16 * w4 + (lane >> 3) + 4 * s4;
          const float4 t0 = *reinterpret_cast<const float4*>(AT + i * kLd + 8 * ch);
          const float4 t1 = *reinterpret_cast<const float4*>(AT + i * kLd + 8 * ch + 4);
          const float tv[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
          uint32_t uw[4], uu[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j0 = 8 * ch + 2 * e;
            const float tu0 = (j0 <= i) ? tv[2 * e] * bj[2 * e] : 0.f;
            const float tu1 = (j0 + 1 <= i) ? tv[2 * e + 1] * bj[2 * e + 1] : 0.f;
            uu[e] = tc::pack2<BF16>(tu0, tu1);
            uw[e] = tc::pack2<BF16>(tu0 * gj[2 * e], tu1 * gj[2 * e + 1]);
          }
          const uint32_t off = tc::sw128_offset(i, ch);
          *reinterpret_cast<uint4*>(rec + kWsTw + off) = make_uint4(uw[0], uw[1], uw[2], uw[3]);
          *reinterpret_cast<uint4*>(rec + kWsTu + off) = make_uint4(uu[0], uu[1], uu[2], uu[3]);
        }
      }
      tc::group_sync(bar, 128);  // AT and the vectors are reused by the next pair
      TRACE1(5);
    }
  }
#ifdef GDN_PREFILL_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 8192) g_cta[blockIdx.x * 5 + 4] = global_timer_ns();
#endif
  if (ht == 64) bulk_wait_all();  // the P tiles have left shared memory
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 64);
#ifdef GDN_PREFILL_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 8192) g_cta[blockIdx.x * 5 + 1] = global_timer_ns();
#endif
}

// ============================================================ state kernel
// One CTA per (batch, value head), 16 warps in three roles:
//   W group  (warps 0-3):  W^T = K^T T_w^T, U^T = V^T T_u^T, the bf16 W^T tile,
//                          refills of V / T_w / T_u;
//   O group  (warps 4-7):  Q rows scaled by gamma_i in place (so that
//                          diag(gamma) Q S and the intra-chunk term accumulate
//                          into one TMEM accumulator), outputs, K/Q/P refills;
//   state    (warps 8-15): the serial chain X -> V' -> dS -> S.
namespace state {
constexpr int kGroupThreads = 128;  // W group, O group
constexpr int kStateThreads = 256;
constexpr int kThreads = 2 * kGroupThreads + kStateThreads;
constexpr int kBarW = 1, kBarState = 2, kBarO = 3;  // named barrier ids

// shared-memory map (byte offsets from a 1024-aligned base)
constexpr uint32_t kKQ = 0;          // 3 slots x [K | Q]: 2 d_k blocks x (K 8 KB + Q 8 KB)
constexpr uint32_t kKQSlot = 32768;
constexpr uint32_t kKQBlock = 16384;
constexpr uint32_t kP = 98304;       // 3 slots x {P tile (8 KB), gamma[64], decay[64]}
constexpr uint32_t kPSlot = 9216;
constexpr uint32_t kV = 126976;      // V tile: 2 d_v blocks x 8 KB (one slot)
constexpr uint32_t kVBlock = 8192;
constexpr uint32_t kTw = 143360;     // T_w tile (8 KB), then T_u (8 KB): one slot
constexpr uint32_t kTu = 151552;
constexpr uint32_t kWQ = 159744;     // W^T, then 2 slots of (diag(gamma) Q)^T: MN-major rows
                                     // d_k, 64 tokens each (16 KB per tile).  W^T and the Q^T
                                     // tile of a chunk form one N = 128 operand whose second
                                     // 64-token block sits 16 KB (slot 0) or 32 KB (slot 1) on
constexpr uint32_t kVP = 208896;     // V'^T, K-major rows d_v               (16 KB)
constexpr uint32_t kBars = 225280;
constexpr uint32_t kSmemBytes = kBars + 256;
constexpr uint32_t kSmemAlloc = kSmemBytes + 1024;
static_assert(kP % 1024 == 0 && kPSlot % 1024 == 0 && kV % 1024 == 0 && kTw % 1024 == 0 &&
              kWQ % 1024 == 0 && kVP % 1024 == 0, "swizzled tiles need 1024-byte alignment");

// TMEM columns
constexpr uint32_t kTmST = 0;    // S^T bf16, packed pairs: 64 columns
constexpr uint32_t kTmW = 64;    // W^T
// 2 slots of 128 columns, each [U^T | O^T]: U^T / V'^T (later V''^T hi | lo as
// bf16 pairs) and the negated output O^T = -(S^T (diag(gamma) Q)^T + V'^T P^T),
// adjacent so that one N = 128 product updates both
constexpr uint32_t kTmUO = 128;
constexpr uint32_t kTmDS = 384, kTmCols = 512;

// mbarrier indices
enum {
  kBarKQP = 0,     // [3] K, Q (TMA), P and the vectors (bulk) of a chunk landed
  kBarTWU = 3,     // V (TMA), T_w | T_u (bulk) of a chunk landed
  kBarHMma = 4,    // W/U MMAs completed
  kBarGo = 5,      // [2] W and O groups -> state: the [W^T | Q^T] tile and U of a
                   //     chunk are ready, and its O slot is clear
  kBarTiles = 7,   // state threads -> MMA thread: V'^T tile and V'' hi / lo written
  kBarSt = 8,      // state threads -> MMA thread: bf16 S^T of the next chunk written
  kBarX = 9,       // V' = U - W S (and the first O term) done
  kBarS2 = 10,     // dS done
  kBarZO = 11,     // [2] O of a chunk complete (its K/Q/P slot is free)
  kBarWT = 13,     // KDA: the W^T tile of a chunk landed (bulk)
  kBarQT = 14,     // KDA: [2] the (Q . exp(G))^T tile of a chunk landed (bulk)
  kNumBars = 16,
};
}  // namespace state

template <bool BF16>
__device__ __forceinline__ uint32_t pack_bits(float lo, float hi) {
  return tc::pack2<BF16>(lo, hi);
}

// dS from one f16 V'' operand (K as f16) instead of bf16 hi + lo halves
constexpr bool kDsSingle = true;

template <bool BF16, bool KDA>
__global__ void __launch_bounds__(state::kThreads, 1)
    state_kernel(const Params p, const __grid_constant__ CUtensorMap map_q,
                 const __grid_constant__ CUtensorMap map_k,
                 const __grid_constant__ CUtensorMap map_v) {
  using namespace state;
  using IO = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBars);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kNumBars);

  const gdn_prefill_args_t& a = p.a;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x;
  const int b = bh / a.Hv, h = bh % a.Hv, hq = h / p.group;
  const int T = a.T;
  const int nchunks = p.nchunks;
  constexpr uint32_t kUnit = KDA ? kKWsUnit : kWsUnit;
  const unsigned char* recs = p.ws + static_cast<size_t>(bh) * nchunks * kUnit;
  auto pvec = [&](int c) {  // GDN {gamma[64], decay[64]}, KDA exp(G_C)[128] of chunk c (in its K/Q/P slot)
    return reinterpret_cast<const float*>(smem + kP + (c % 3) * kPSlot + 8192);
  };

  if (warp == 0) tc::tmem_alloc(tmem_holder, kTmCols);
  if (tid == 0) {
    for (int i = 0; i < 3; ++i) mbar_init(&bars[kBarKQP + i], 1);
    mbar_init(&bars[kBarTWU], 1);
    mbar_init(&bars[kBarHMma], 1);
    for (int i = 0; i < 2; ++i) mbar_init(&bars[kBarGo + i], 2 * kGroupThreads);
    mbar_init(&bars[kBarTiles], kStateThreads);
    mbar_init(&bars[kBarSt], kStateThreads);
    mbar_init(&bars[kBarX], 1);
    mbar_init(&bars[kBarS2], 1);
    mbar_init(&bars[kBarZO], 1);
    mbar_init(&bars[kBarZO + 1], 1);
    mbar_init(&bars[kBarWT], 1);
    mbar_init(&bars[kBarQT], 1);
    mbar_init(&bars[kBarQT + 1], 1);
    fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
  constexpr uint32_t kIdW = tc::idesc_f16(128, 64, true, false, BF16);
  constexpr uint32_t kIdXZ = tc::idesc_f16(128, 128, false, true, BF16, true);
  constexpr uint32_t kIdOIneg = tc::idesc_f16(128, 64, false, false, BF16, true);
  // KDA: dS^T = V'^T (K . exp(G_C - G)) takes f16 operands (the decayed keys
  // keep 11 mantissa bits; V' enters as f16 hi + lo)
  constexpr uint32_t kIdDS = tc::idesc_f16(128, 128, false, true, (KDA || kDsSingle) ? false : BF16);

  // GDN: K, Q (TMA), P and vectors (bulk) of chunk n into slot n % 3.
  // KDA: the decayed keys (in the K tile places), P and exp(G_C), all bulk.
  auto issue_kqp = [&](int n) {
    const int slot = n % 3;
    uint64_t* bar = &bars[kBarKQP + slot];
    const unsigned char* rec = recs + static_cast<size_t>(n) * kUnit;
    if constexpr (KDA) {
      mbar_arrive_expect_tx(bar, 2 * 8192 + 8192 + 512);
#pragma unroll
      for (int blk = 0; blk < 2; ++blk)
        bulk_g2s(smem + kKQ + slot * kKQSlot + blk * kKQBlock, rec + kKWsKd + blk * 8192, 8192, bar);
      bulk_g2s(smem + kP + slot * kPSlot, rec + kKWsP, 8192, bar);
      bulk_g2s(smem + kP + slot * kPSlot + 8192, rec + kKWsVec, 512, bar);
    } else {
      mbar_arrive_expect_tx(bar, 4 * 8192 + 8192 + 512);
      const int t0 = n * kC;
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
        unsigned char* kq = smem + kKQ + slot * kKQSlot + blk * kKQBlock;
        tc::tma_load_4d(kq, &map_k, blk * 64, hq, t0, b, bar);
        tc::tma_load_4d(kq + 8192, &map_q, blk * 64, hq, t0, b, bar);
      }
      bulk_g2s(smem + kP + slot * kPSlot, rec + kWsP, 8192, bar);
      bulk_g2s(smem + kP + slot * kPSlot + 8192, rec + kWsVec, 512, bar);
    }
  };
  auto issue_twu = [&](int n) {  // V (TMA), T_w | T_u (GDN) or T_u (KDA) (bulk) of chunk n
    uint64_t* bar = &bars[kBarTWU];
    mbar_arrive_expect_tx(bar, 2 * 8192 + (KDA ? 8192 : 16384));
    const int t0 = n * kC;
#pragma unroll
    for (int blk = 0; blk < 2; ++blk)
      tc::tma_load_4d(smem + kV + blk * kVBlock, &map_v, blk * 64, h, t0, b, bar);
    if constexpr (KDA)
      bulk_g2s(smem + kTu, recs + static_cast<size_t>(n) * kUnit + kKWsTu, 8192, bar);
    else
      bulk_g2s(smem + kTw, recs + static_cast<size_t>(n) * kUnit + kWsTw, 16384, bar);
  };
  // KDA: the W^T tile of chunk n (into kWQ, after X of chunk n - 1 read it)
  // and the (Q . exp(G))^T tile of chunk n (into Q^T slot n & 1)
  auto issue_wt = [&](int n) {
    mbar_arrive_expect_tx(&bars[kBarWT], 16384);
    bulk_g2s(smem + kWQ, recs + static_cast<size_t>(n) * kUnit + kKWsWT, 16384, &bars[kBarWT]);
  };
  auto issue_qt = [&](int n) {
    uint64_t* bar = &bars[kBarQT + (n & 1)];
    mbar_arrive_expect_tx(bar, 16384);
    bulk_g2s(smem + kWQ + 16384 * (1 + (n & 1)), recs + static_cast<size_t>(n) * kUnit + kKWsQT, 16384, bar);
  };
  // Launched as a programmatic dependent of the intra kernel: everything up
  // to here (and the state warps' initial-state load) overlaps its tail; the
  // workspace and the inputs are read only after pdl_wait().
  if (tid == 2 * kGroupThreads) {
    pdl_wait();
    for (int n = 0; n < 3 && n < nchunks; ++n) issue_kqp(n);
    issue_twu(0);
    if constexpr (KDA) {
      for (int n = 0; n < 2 && n < nchunks; ++n) issue_qt(n);
    }
  }

  if (warp < 4) {
    // ================================================================ W group
    asm volatile("setmaxnreg.dec.sync.aligned.u32 88;" ::: "memory");
    pdl_wait();
    const int k = warp * 32 + lane;  // W^T row (d_k) this thread converts
    bool ok = true;
    if constexpr (KDA) {
      // KDA: W^T arrives precomputed (bulk); only U^T = V^T T_u^T is formed here
      for (int c = 0; c < nchunks; ++c) {
        const int slot = c & 1;
        const uint32_t tmu = tmem + kTmUO + slot * 128;
        if (!group_wait(&bars[kBarTWU], c & 1, kBarW, kGroupThreads)) { ok = false; break; }
        // the U slot was last used by chunk c - 2 and the W^T tile by X of c - 1
        if (c >= 1 && !group_wait(&bars[kBarX], (c - 1) & 1, kBarW, kGroupThreads)) { ok = false; break; }
        TRACE(c, 0);
        if (tid == 0) {
          issue_wt(c);
          tc::fence_after_sync();
#pragma unroll
          for (int s = 0; s < 4; ++s)
            tc::mma(tmu, tc::mnmajor_desc(sb + kV, kVBlock, s), tc::kmajor_desc(sb + kTu, 0, s), kIdW, s > 0);
          tc::commit(&bars[kBarHMma]);
        }
        if (!group_wait(&bars[kBarHMma], c & 1, kBarW, kGroupThreads)) { ok = false; break; }
        if (tid == 0 && c + 1 < nchunks) issue_twu(c + 1);  // V / T_u slot is free again
        if (!group_wait(&bars[kBarWT], c & 1, kBarW, kGroupThreads)) { ok = false; break; }
        TRACE(c, 1);
        tc::fence_before_sync();
        mbar_arrive(&bars[kBarGo + slot]);
        TRACE(c, 2);
      }
    } else for (int c = 0; c < nchunks; ++c) {
      const int slot = c & 1;
      const uint32_t kq = sb + kKQ + (c % 3) * kKQSlot;
      const uint32_t tmu = tmem + kTmUO + slot * 128;
      if (!group_wait(&bars[kBarKQP + c % 3], (c / 3) & 1, kBarW, kGroupThreads)) { ok = false; break; }
      if (!group_wait(&bars[kBarTWU], c & 1, kBarW, kGroupThreads)) { ok = false; break; }
      // the U slot was last used by chunk c - 2 (its dS MMA precedes X of c - 1)
      // and the W^T tile by X of chunk c - 1
      if (c >= 1 && !group_wait(&bars[kBarX], (c - 1) & 1, kBarW, kGroupThreads)) { ok = false; break; }
      TRACE(c, 0);
      if (tid == 0) {  // W^T = K^T T_w^T, U^T = V^T T_u^T
        tc::fence_after_sync();
#pragma unroll
        for (int s = 0; s < 4; ++s)
          tc::mma(tmem + kTmW, tc::mnmajor_desc(kq, kKQBlock, s), tc::kmajor_desc(sb + kTw, 0, s), kIdW, s > 0);
#pragma unroll
        for (int s = 0; s < 4; ++s)
          tc::mma(tmu, tc::mnmajor_desc(sb + kV, kVBlock, s), tc::kmajor_desc(sb + kTu, 0, s), kIdW, s > 0);
        tc::commit(&bars[kBarHMma]);
      }
      if (!group_wait(&bars[kBarHMma], c & 1, kBarW, kGroupThreads)) { ok = false; break; }
      tc::fence_after_sync();
      if (tid == 0 && c + 1 < nchunks) issue_twu(c + 1);  // V / T_w / T_u slot is free again
      if (kDsSingle && BF16) {
        // the W product has read the K tile; dS reads it as f16 (bf16 -> f16 is
        // exact for |k| >= 2^-14; below that it becomes subnormal)
        unsigned char* kt = smem + kKQ + (c % 3) * kKQSlot;
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const int idx = v * kGroupThreads + tid;  // 16-byte piece of the 2 x 8 KB K tile
          uint4* pp = reinterpret_cast<uint4*>(kt + (idx >> 9) * kKQBlock + (idx & 511) * 16);
          uint4 x = *pp;
          uint32_t* w = reinterpret_cast<uint32_t*>(&x);
#pragma unroll
          for (int e = 0; e < 4; ++e) w[e] = tc::pack2<false>(tc::unpack_lo<true>(w[e]), tc::unpack_hi<true>(w[e]));
          *pp = x;
        }
      }
      TRACE(c, 1);
#pragma unroll
      for (int ih = 0; ih < 2; ++ih) {  // W^T -> bf16 tile, MN-major rows d_k, tokens [32 ih, +32)
        float r[32];
        tc::tmem_ld16(tmem + lane_base + kTmW + ih * 32, *reinterpret_cast<float(*)[16]>(r));
        tc::tmem_ld16(tmem + lane_base + kTmW + ih * 32 + 16, *reinterpret_cast<float(*)[16]>(r + 16));
        tc::tmem_wait_ld();
        store_row16<BF16>(sb + kWQ, k, ih * 4, r);
        store_row16<BF16>(sb + kWQ, k, ih * 4 + 2, r + 16);
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      mbar_arrive(&bars[kBarGo + slot]);
      TRACE(c, 2);
    }
    if (!ok && tid == 0) report(a.status, GDN_DEVERR_MMA_TIMEOUT);
  } else if (warp < 8) {
    // ================================================================ O group
    asm volatile("setmaxnreg.dec.sync.aligned.u32 88;" ::: "memory");
    pdl_wait();
    const int ot = tid - kGroupThreads;  // 0..127
    const int dv = (warp & 3) * 32 + lane;
    IO* o = static_cast<IO*>(a.o);
    auto zero_o = [&](int slot) {  // the O product of the next chunk in this slot starts from 0
      uint32_t z[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) z[e] = 0u;
#pragma unroll
      for (int q = 0; q < 4; ++q) tc::tmem_st16(tmem + kTmUO + slot * 128 + 64 + lane_base + q * 16, z);
      tc::tmem_wait_st();
      tc::fence_before_sync();
    };
    // (diag(gamma) Q)^T of chunk c into Q^T slot c & 1: 8 x 8 blocks moved
    // with ldmatrix.trans / stmatrix.  Warp w handles d_k blocks 4w..4w+3,
    // four 8-token blocks per instruction.
    auto scale_q = [&](int c) -> bool {
      if (!group_wait(&bars[kBarKQP + c % 3], (c / 3) & 1, kBarO, kGroupThreads)) return false;
      const float* gam = pvec(c);
      const int w = warp & 3, m = lane >> 3, r8 = lane & 7;
      const uint32_t qslot = sb + kKQ + (c % 3) * kKQSlot + 8192;
      const uint32_t qt = sb + kWQ + 16384 * (1 + (c & 1));
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kc = w * 4 + j;  // d_k rows 8 kc .. 8 kc + 7 (K block kc / 8)
        const uint32_t src = qslot + (kc >> 3) * kKQBlock;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t v[4];
          tc::ldsm_x4_trans(src + tc::sw128_offset(8 * (4 * hh + m) + r8, kc & 7), v);
#pragma unroll
          for (int mm = 0; mm < 4; ++mm) {
            const float2 g2 = *reinterpret_cast<const float2*>(gam + 8 * (4 * hh + mm) + 2 * (lane & 3));
            v[mm] = tc::pack2<BF16>(g2.x * tc::unpack_lo<BF16>(v[mm]), g2.y * tc::unpack_hi<BF16>(v[mm]));
          }
          tc::stsm_x4(qt + tc::sw128_offset(8 * kc + r8, 4 * hh + m), v);
        }
      }
      tc::fence_proxy_async();
      return true;
    };
    // outputs o[t0 + i][dv] = -scale O[dv][i] (O holds the negated product)
    // of chunk c, after which the O slot is cleared and the go of chunk c + 2
    // (its scaled Q^T tile and this cleared slot) is announced.  The outputs
    // are staged, row-major, in the Q tile of K/Q/P slot (c + 2) % 3, which is
    // no longer needed once its scaled copy exists (or holds the finished
    // chunk c - 1), and then written with coalesced 16-byte stores.
    auto outputs = [&](int c) -> bool {
      if (!group_wait(&bars[kBarZO + (c & 1)], (c >> 1) & 1, kBarO, kGroupThreads)) return false;
      tc::fence_after_sync();
      if (ot == 0 && c + 3 < nchunks) issue_kqp(c + 3);  // every MMA of chunk c is done
      if constexpr (KDA) {
        if (ot == 0 && c + 2 < nchunks) issue_qt(c + 2);  // Q^T slot c & 1 was last read by X of c
      } else {
        if (c + 2 < nchunks && !scale_q(c + 2)) return false;
      }
      tc::group_sync(kBarO, kGroupThreads);  // every warp has read the Q tile reused below
      const uint32_t tmo = tmem + kTmUO + (c & 1) * 128 + 64;
      unsigned char* stage = smem + kKQ + ((c + 2) % 3) * kKQSlot + 8192;  // + (dv / 64) * kKQBlock
      const float ns = -a.scale;
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        float r[32];
        tc::tmem_ld16(tmo + lane_base + hb * 32, *reinterpret_cast<float(*)[16]>(r));
        tc::tmem_ld16(tmo + lane_base + hb * 32 + 16, *reinterpret_cast<float(*)[16]>(r + 16));
        tc::tmem_wait_ld();
        if (hb == 1) {
          zero_o(c & 1);
          mbar_arrive(&bars[kBarGo + (c & 1)]);  // go of chunk c + 2
        }
        IO* st_col = reinterpret_cast<IO*>(stage + (dv >> 6) * kKQBlock) + (dv & 63);
#pragma unroll
        for (int i = 0; i < 32; ++i) st_col[(hb * 32 + i) * 64] = from_f32<IO>(ns * r[i]);
      }
      tc::group_sync(kBarO, kGroupThreads);
      const int t0 = c * kC;
#pragma unroll
      for (int rr = 0; rr < 8; ++rr) {  // 64 rows x 256 B = 1024 16-byte pieces
        const int piece = rr * kGroupThreads + ot;
        const int i = piece >> 4, col = (piece & 15) * 8;
        if (t0 + i < T) {
          const uint4 v = *reinterpret_cast<const uint4*>(stage + (col >> 6) * kKQBlock + i * 128 + (col & 63) * 2);
          *reinterpret_cast<uint4*>(o + ((static_cast<int64_t>(b) * T + t0 + i) * a.Hv + h) * kD + col) = v;
        }
      }
      tc::group_sync(kBarO, kGroupThreads);  // the staging tile may be refilled
      return true;
    };
    zero_o(0);
    zero_o(1);
    bool ok = true;
    for (int c = 0; c < 2 && c < nchunks && ok; ++c) {
      if constexpr (!KDA) ok = scale_q(c);  // KDA: the scaled Q^T tiles arrive by bulk copy
      if (ok) {
        tc::fence_before_sync();
        mbar_arrive(&bars[kBarGo + c]);
      }
    }
    for (int c = 0; c < nchunks && ok; ++c) {
      if (!outputs(c)) { ok = false; break; }
      TRACE(c, 3);
    }
    if (!ok && ot == 0) report(a.status, GDN_DEVERR_MMA_TIMEOUT);
  } else {
    // ================================================================ state
    asm volatile("setmaxnreg.inc.sync.aligned.u32 168;" ::: "memory");
    const int st = tid - 2 * kGroupThreads;  // 0..255
    const int quarter = warp & 3, half = (warp - 8) >> 2;
    const int dv = quarter * 32 + lane;
    const int k0 = half * 64;
    const size_t state_off = static_cast<size_t>(bh) * kD * kD;
    float S[64];
#pragma unroll
    for (int j = 0; j < 64; ++j)
      S[j] = a.initial_state ? a.initial_state[state_off + static_cast<size_t>(k0 + j) * kD + dv] : 0.f;
    // the initial state is not an output of the intra kernel (whose own
    // predecessor completed before it let this kernel start)
    pdl_wait();
    auto write_st = [&]() {  // bf16 S^T into TMEM: lane dv, packed d_k pairs
#pragma unroll
      for (int cb = 0; cb < 2; ++cb) {
        uint32_t u[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) u[e] = pack_bits<BF16>(S[cb * 32 + 2 * e], S[cb * 32 + 2 * e + 1]);
        tc::tmem_st16(tmem + lane_base + kTmST + half * 32 + cb * 16, u);
      }
      tc::tmem_wait_st();
      tc::fence_before_sync();
    };
    write_st();
    tc::group_sync(kBarState, kStateThreads);
    // Only the MMA thread (st == 0) waits for the other groups and for the
    // state threads' writes (mbarriers); all threads meet in a barrier vote
    // only where they need an MMA result (X and dS), and the MMA thread joins
    // those votes with its own waits' outcome.
    bool ok = true;
    for (int c = 0; c < nchunks; ++c) {
      const int slot = c & 1;
      const uint32_t kq = sb + kKQ + (c % 3) * kKQSlot;
      const uint32_t pt = sb + kP + (c % 3) * kPSlot;
      const uint32_t tmu = tmem + kTmUO + slot * 128;
      const uint32_t tmo = tmu + 64;
      bool mine = true;
      if (st == 0) {  // [V'^T | O^T] = [U^T | 0] - S^T [W^T | (diag(gamma) Q)^T]  (A = S^T from TMEM)
        mine = (c == 0 || mbar_wait_bounded(&bars[kBarSt], (c - 1) & 1)) &&
               mbar_wait_bounded(&bars[kBarGo + slot], (c >> 1) & 1) &&
               (!KDA || mbar_wait_bounded(&bars[kBarQT + slot], (c >> 1) & 1));
        TRACE(c, 4);
        if (mine) {
          tc::fence_after_sync();
#pragma unroll
          for (int s = 0; s < 8; ++s)
            tc::mma_tmem_a(tmu, tmem + kTmST + s * 8, tc::mnmajor_desc(sb + kWQ, 16384 * (1 + slot), s),
                           kIdXZ, true);
          tc::commit(&bars[kBarX]);
        }
      }
      const float* vc = pvec(c);
      if (!group_wait(&bars[kBarX], c & 1, kBarState, kStateThreads, !mine)) { ok = false; break; }
      tc::fence_after_sync();
      const float gC = KDA ? 0.f : vc[kC - 1];
      TRACE(c, 5);
      {  // V' (TMEM) -> bf16 V'^T tile; V'' = V' exp(G_C - G_j) -> bf16 hi / lo
         // written back over the thread's own V' columns: for its 32 tokens,
         // hi in the first 16 packed columns and lo in the next 16
        float u[32];
        tc::tmem_ld16(tmu + lane_base + half * 32, *reinterpret_cast<float(*)[16]>(u));
        tc::tmem_ld16(tmu + lane_base + half * 32 + 16, *reinterpret_cast<float(*)[16]>(u + 16));
        tc::tmem_wait_ld();
#pragma unroll
        for (int cb = 0; cb < 2; ++cb) {
          uint32_t wp[8], wh[8], wl[8];
          const float4* dec4 = reinterpret_cast<const float4*>(vc + 64 + half * 32 + cb * 16);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const float4 d = dec4[q4];
            const float dd[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
            for (int e2 = 0; e2 < 2; ++e2) {
              const int e = q4 * 2 + e2;
              const float u0 = u[cb * 16 + 2 * e], u1 = u[cb * 16 + 2 * e + 1];
              wp[e] = tc::pack2<BF16>(u0, u1);
              if constexpr (kDsSingle) {  // one f16 operand: V' (KDA) or V'' (GDN)
                wh[e] = KDA ? tc::pack2<false>(u0, u1) : tc::pack2<false>(u0 * dd[2 * e2], u1 * dd[2 * e2 + 1]);
                wl[e] = 0u;
              } else if constexpr (KDA) {  // the decay sits in the keys; V' as f16 hi + lo
                const uint32_t hw = tc::pack2<false>(u0, u1);
                wh[e] = hw;
                wl[e] = tc::pack2<false>(u0 - tc::unpack_lo<false>(hw), u1 - tc::unpack_hi<false>(hw));
              } else {
                const float v0 = u0 * dd[2 * e2], v1 = u1 * dd[2 * e2 + 1];
                const uint32_t hw = tc::pack2<BF16>(v0, v1);
                wh[e] = hw;
                wl[e] = tc::pack2<BF16>(v0 - tc::unpack_lo<BF16>(hw), v1 - tc::unpack_hi<BF16>(hw));
              }
            }
          }
          const int ch = half * 4 + cb * 2;
#pragma unroll
          for (int k2 = 0; k2 < 2; ++k2)
            tc::sts128(sb + kVP + tc::sw128_offset(dv, ch + k2), wp[4 * k2], wp[4 * k2 + 1],
                       wp[4 * k2 + 2], wp[4 * k2 + 3]);
          // this thread's V' columns were loaded (tcgen05.wait::ld) before the overwrite
          tc::tmem_st8(tmu + lane_base + half * 32 + cb * 8, wh);
          if (!kDsSingle) tc::tmem_st8(tmu + lane_base + half * 32 + 16 + cb * 8, wl);
        }
        tc::tmem_wait_st();
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      mbar_arrive(&bars[kBarTiles]);
      TRACE(c, 6);
      if (st == 0) {  // dS^T = V''hi^T K + V''lo^T K (A from TMEM), then O^T -= V'^T P^T
        mine = mbar_wait_bounded(&bars[kBarTiles], c & 1);
        if (mine) {
          tc::fence_after_sync();
#pragma unroll
          for (int s = 0; s < 4; ++s)  // tokens [16 s, 16 s + 16): hi of half s / 2
            tc::mma_tmem_a(tmem + kTmDS, tmu + (s >> 1) * 32 + (s & 1) * 8, tc::mnmajor_desc(kq, kKQBlock, s),
                           kIdDS, s > 0);
          if (!kDsSingle) {
#pragma unroll
            for (int s = 0; s < 4; ++s)
              tc::mma_tmem_a(tmem + kTmDS, tmu + (s >> 1) * 32 + 16 + (s & 1) * 8,
                             tc::mnmajor_desc(kq, kKQBlock, s), kIdDS, true);
          }
          tc::commit(&bars[kBarS2]);
#pragma unroll
          for (int s = 0; s < 4; ++s)
            tc::mma(tmo, tc::kmajor_desc(sb + kVP, 0, s), tc::kmajor_desc(pt, 0, s), kIdOIneg, true);
          tc::commit(&bars[kBarZO + slot]);
        }
      }
      // dS done, and with it the earlier X / O product that read the old S^T
      // (tcgen05 operations of one thread complete in order)
      if (!group_wait(&bars[kBarS2], c & 1, kBarState, kStateThreads, !mine)) { ok = false; break; }
      tc::fence_after_sync();
      TRACE(c, 7);
      {  // S <- gamma_C S + dS ; bf16 S^T back into TMEM for the next chunk
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          float r[32];
          tc::tmem_ld16(tmem + lane_base + kTmDS + half * 64 + hb * 32, *reinterpret_cast<float(*)[16]>(r));
          tc::tmem_ld16(tmem + lane_base + kTmDS + half * 64 + hb * 32 + 16,
                        *reinterpret_cast<float(*)[16]>(r + 16));
          tc::tmem_wait_ld();
          if constexpr (KDA) {  // per-row decay exp(G_C)[d_k]
#pragma unroll
            for (int j4 = 0; j4 < 32; j4 += 4) {
              const float4 g4 = *reinterpret_cast<const float4*>(vc + k0 + hb * 32 + j4);
              S[hb * 32 + j4] = fmaf(g4.x, S[hb * 32 + j4], r[j4]);
              S[hb * 32 + j4 + 1] = fmaf(g4.y, S[hb * 32 + j4 + 1], r[j4 + 1]);
              S[hb * 32 + j4 + 2] = fmaf(g4.z, S[hb * 32 + j4 + 2], r[j4 + 2]);
              S[hb * 32 + j4 + 3] = fmaf(g4.w, S[hb * 32 + j4 + 3], r[j4 + 3]);
            }
          } else {
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) S[hb * 32 + jj] = fmaf(gC, S[hb * 32 + jj], r[jj]);
          }
        }
        write_st();
      }
      mbar_arrive(&bars[kBarSt]);
      TRACE(c, 8);
    }
    if (ok && nchunks > 0) {
#pragma unroll
      for (int j = 0; j < 64; ++j)
        a.final_state[state_off + static_cast<size_t>(k0 + j) * kD + dv] = S[j];
    }
    if (!ok && st == 0) report(a.status, GDN_DEVERR_MMA_TIMEOUT);
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, kTmCols);
}

// ============================================================ KDA intra kernel
// KDA (per-channel log gate g[t][c]) version of the intra kernel.  With G the
// in-chunk cumulative log gate per channel, every pairwise factor
// exp(G_ic - G_jc) now depends on the channel, so the decays go into the MMA
// operands instead of scaling the product:
//   A_ij / beta_i = sum_c [k_ic exp(G_ic - r_c)] [k_jc exp(r_c - G_jc)]
// for any reference point r.  Fast path (every |G| <= 80 in the chunk): r = 0,
// so the left factors are K . exp(G) and Q . exp(G) — the operands the W
// product and the state pass need anyway — and one M = 128, N = 64 MMA gives
// all A and P rows; every factor lies in [exp(-80), exp(80)], finite in bf16.
// Slow path (stronger decays): per row block I (tokens 16 I .. 16 I + 15)
// r = G at token 16 I, which keeps the left factors <= 1 and the right ones
// <= 1 below the diagonal block; one MMA per row block (N = 16 (I + 1)), and
// the diagonal blocks, where the factored form could overflow, summed
// directly from the gates.  The remaining operands of the state pass (W^T,
// (Q . exp(G))^T, the decayed keys K . exp(G_C - G) and exp(G_C)) are formed
// here too, so the state kernel's per-chunk work is the GDN one.
namespace kintra {
constexpr int kThreads = 256;
constexpr uint32_t kKQ = 0;            // [K | Q] per d_k block (2 x 16 KB), scaled in place
constexpr uint32_t kKQBlock = 16384;
constexpr uint32_t kAT = 0;            // A -> T over the K/Q tiles once the products are done
constexpr uint32_t kMs = 64 * kLd * 4; // 17408: solver scratch (4608 B), likewise
constexpr uint32_t kKn = 32768;        // right factors of row block I: 16 (I + 1) rows each
constexpr uint32_t kKnBytes = 40960;
constexpr int kGLd = 130;              // slow path: G [64][kGLd] fp32 over the right factors
constexpr uint32_t kGs = kKn;
constexpr uint32_t kGTile = kKn;       // the raw gate tile (up to 32 KB), consumed before the build
constexpr uint32_t kKg = kKn + kKnBytes;  // 73728: K . exp(G), 2 d_k blocks x 8 KB
constexpr uint32_t kTu = kKg + 16384;     // 90112: P staging, then T_u
constexpr uint32_t kBeta = kTu + 8192;    // 98304: beta[64]
constexpr uint32_t kGb = kBeta + 256;     // G at tokens 0, 16, 32, 48 and 63, per channel [5][128]
constexpr uint32_t kPart = kGb + 5 * 128 * 4;   // per-block gate sums [4][128]
constexpr uint32_t kBars = kPart + 4 * 128 * 4;
constexpr uint32_t kSmemBytes = kBars + 64;
constexpr uint32_t kSmemAlloc = kSmemBytes + 1024;
constexpr uint32_t kTmCols = 256;      // A/P products at 8 I (I + 1) (160 columns), W^T at 192
constexpr uint32_t kTmW = 192;
constexpr uint32_t kTmFast = 96;       // fast path: the one 64-column product (row block 3's columns)
constexpr uint32_t kATFast = kKn;      // fast path: A -> T and the solver scratch over the
                                       // consumed right factors, then the Q^T staging tile
constexpr uint32_t kQTStage = kKn + 24576;
// compact fast-path-only map (kda_intra_fast): [K | Q] 32 KB, then R (32 KB):
// the raw gate tile, then K . exp(-G), then A -> T and the solver scratch;
// P staging / T_u at the end of R; the vectors; the barriers
constexpr uint32_t kFoR = 32768;
constexpr uint32_t kFoTu = kFoR + 23552;
constexpr uint32_t kFoVec = 65536;
constexpr uint32_t kFoBars = kFoVec + 256 + 5 * 128 * 4 + 4 * 128 * 4;
constexpr uint32_t kFoSmemAlloc = kFoBars + 64 + 1024;
constexpr uint32_t kFoTmCols = 128;    // the A/P product at 0, W^T at 64
static_assert(kFoR + 64 * kLd * 4 + 4608 <= kFoTu && kFoTu + 8192 <= kFoVec && kFoTu % 1024 == 0,
              "compact smem map");
__host__ __device__ constexpr uint32_t kn_off(int I) { return 2048u * I * (I + 1); }
__host__ __device__ constexpr uint32_t kn_blk(int I) { return 2048u * (I + 1); }
static_assert(kMs + 4608 <= kKn && 64 * kGLd * 4 <= kKnBytes && kn_off(4) == kKnBytes, "smem map");
static_assert(kATFast + kMs + 4608 <= kQTStage && kQTStage + 16384 <= kKn + kKnBytes &&
              kQTStage % 1024 == 0, "fast-path smem map");
}  // namespace kintra

// One (batch, value head, chunk) unit of the KDA intra kernel.  FO selects the
// compact fast-path-only variant (three CTAs per SM); it returns false, having
// written nothing, for a chunk whose |G| exceeds the fast path's range.  The
// other variant (FO = false) runs the slow path for such chunks.  `par` is the
// mbarrier phase of this unit (units of one CTA alternate).
template <bool BF16, bool FO>
__device__ __forceinline__ bool kda_unit(const Params& p, const CUtensorMap& map_q, const CUtensorMap& map_k,
                                         const CUtensorMap& map_g, int unit, uint32_t par,
                                         unsigned char* smem, uint64_t* bars, uint32_t tmem) {
  using namespace kintra;
  using IO = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  const uint32_t sb = smem_u32(smem);
  const gdn_prefill_args_t& a = p.a;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int per_c = a.B * a.Hv;
  const int c = p.nchunks - 1 - unit / per_c;
  const int bh = unit % per_c;
  const int b = bh / a.Hv, h = bh % a.Hv, hq = h / p.group;
  const int T = a.T, t0 = c * kC;
  unsigned char* rec = p.ws + (static_cast<size_t>(bh) * p.nchunks + c) * kKWsUnit;
  // build-phase role: token block J, d_k block kb, channels ch, ch + 1
  const int J = warp >> 1, kb = warp & 1;
  const int ch = kb * 64 + 2 * lane;

  KTRACE(0);
  // smem map of this kernel variant (FO: the compact fast-path-only map)
  constexpr uint32_t oGT = FO ? kFoR : kGTile;          // raw gate tile
  constexpr uint32_t oKnF = FO ? kFoR : kKn + kn_off(3);  // fast path: K . exp(-G), d_k block stride 8 KB
  constexpr uint32_t oATF = FO ? kFoR : kATFast;        // fast path: A -> T, then the solver scratch
  constexpr uint32_t oTu = FO ? kFoTu : kTu;            // P staging, then T_u
  constexpr uint32_t oBeta = FO ? kFoVec : kBeta;
  constexpr uint32_t oGb = oBeta + 256, oPart = oGb + 5 * 128 * 4;
  constexpr uint32_t oTmFast = FO ? 0 : kTmFast, oTmW = FO ? 64 : kTmW;
  static_assert(kn_blk(3) == 8192, "fast right-factor tile: 64 rows per d_k block");
  // raw gates of this thread's 16 tokens and 2 channels (converted at first use)
  auto load_gates = [&](uint32_t (&g0)[16], uint32_t (&g1)[16]) {
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      g0[r] = 0u;  // padded tokens: no decay
      g1[r] = 0u;
      const int t = t0 + 16 * J + r;
      if (t < T) {
        const int64_t gi = ((static_cast<int64_t>(b) * T + t) * a.Hv + h) * kD + ch;
        if (a.g_dtype == GDN_DT_F32) {
          const uint2 u = __ldg(reinterpret_cast<const uint2*>(a.g) + (gi >> 1));
          g0[r] = u.x;
          g1[r] = u.y;
        } else {
          g0[r] = __ldg(reinterpret_cast<const uint32_t*>(a.g) + (gi >> 1));
        }
      }
    }
  };
  uint32_t braw = 0u;
  if (tid < kC && t0 + tid < T) {
    const int64_t bi = (static_cast<int64_t>(b) * T + t0 + tid) * a.Hv + h;
    braw = a.beta_dtype == GDN_DT_F32 ? __ldg(reinterpret_cast<const uint32_t*>(a.beta) + bi)
                                      : __ldg(reinterpret_cast<const unsigned short*>(a.beta) + bi);
  }
  auto gate = [&](uint32_t raw, bool hi) -> float {
    if (a.g_dtype == GDN_DT_F32) return __uint_as_float(raw);
    const uint32_t bits = hi ? (raw >> 16) : (raw & 0xFFFFu);
    if (a.g_dtype == GDN_DT_BF16) return __uint_as_float(bits << 16);
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits)));
  };

  __syncthreads();  // the previous unit of this CTA is done with shared memory
  const bool gf32 = a.g_dtype == GDN_DT_F32;
  if (tid == 0) {  // K, Q tiles and the gate tile [64 tokens][128 channels] (zero past T)
    mbar_arrive_expect_tx(&bars[0], 4 * 8192 + kC * kD * (gf32 ? 4 : 2));
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
      unsigned char* kq = smem + kKQ + blk * kKQBlock;
      tc::tma_load_4d(kq, &map_k, blk * 64, hq, t0, b, &bars[0]);
      tc::tma_load_4d(kq + 8192, &map_q, blk * 64, hq, t0, b, &bars[0]);
    }
    tc::tma_load_4d(smem + oGT, &map_g, 0, h, t0, b, &bars[0]);
  }
  KTRACE(11);
  bool ok = !named_barrier_or(1, kThreads, (lane == 0) && !mbar_wait_bounded(&bars[0], par));
  KTRACE(12);
  uint32_t gr0[16], gr1[16];  // raw gates of this thread's tokens and channels
#pragma unroll
  for (int r = 0; r < 16; ++r) {
    const int i = 16 * J + r;
    if (gf32) {
      const uint2 u = *reinterpret_cast<const uint2*>(smem + oGT + (i * kD + ch) * 4);
      gr0[r] = u.x;
      gr1[r] = u.y;
    } else {
      gr0[r] = *reinterpret_cast<const uint32_t*>(smem + oGT + (i * kD + ch) * 2);
      gr1[r] = 0u;
    }
  }

  // ---- in-chunk cumulative log gate per channel
  float* sBeta = reinterpret_cast<float*>(smem + oBeta);
  float* sGb = reinterpret_cast<float*>(smem + oGb);
  float* sPart = reinterpret_cast<float*>(smem + oPart);
  // in-block inclusive prefix sums of the raw gates (channels ch, ch + 1)
  auto block_scan = [&](const uint32_t (&g0)[16], const uint32_t (&g1)[16], float (&o0)[16], float (&o1)[16]) {
    float run0 = 0.f, run1 = 0.f;
    const bool f32 = a.g_dtype == GDN_DT_F32;
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      run0 += gate(g0[r], false);
      run1 += f32 ? gate(g1[r], false) : gate(g0[r], true);
      o0[r] = run0;
      o1[r] = run1;
    }
  };
  // G of the earlier blocks of the chunk (from the block sums in sPart)
  auto block_offset = [&](float& o0, float& o1) {
    o0 = 0.f;
    o1 = 0.f;
    for (int jb = 0; jb < J; ++jb) {
      const float2 pp = *reinterpret_cast<const float2*>(sPart + jb * 128 + ch);
      o0 += pp.x;
      o1 += pp.y;
    }
  };
  float G0[16], G1[16];
  {
    block_scan(gr0, gr1, G0, G1);
    *reinterpret_cast<float2*>(sPart + J * 128 + ch) = make_float2(G0[15], G1[15]);
    KTRACE(13);
    if (tid < kC) {
      sBeta[tid] = a.beta_dtype == GDN_DT_F32   ? __uint_as_float(braw)
                   : a.beta_dtype == GDN_DT_BF16 ? __uint_as_float(braw << 16)
                                                 : __half2float(__ushort_as_half(static_cast<unsigned short>(braw)));
    }
  }
  __syncthreads();
  bool in_range = true;
  {
    float o0, o1;
    block_offset(o0, o1);
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      G0[r] += o0;
      G1[r] += o1;
      in_range = in_range && fabsf(G0[r]) <= 80.f && fabsf(G1[r]) <= 80.f;
    }
    *reinterpret_cast<float2*>(sGb + J * 128 + ch) = make_float2(G0[0], G1[0]);
    if (J == 3) *reinterpret_cast<float2*>(sGb + 4 * 128 + ch) = make_float2(G0[15], G1[15]);
  }
  // also publishes sGb / sBeta.  The compact variant defers a chunk outside
  // the fast path's range to the other variant, which runs only the slow path.
  if (FO) {
    if (__syncthreads_or(ok && !in_range)) return false;
  } else {
    __syncthreads();
  }
  constexpr bool fast = FO;
  KTRACE(1);

  // ---- scaled operands
  // Fast path: one reference point for the whole chunk,
  //   A/P = [K . exp(G); Q . exp(G)] (K . exp(-G))^T,
  // with every factor in [exp(-80), exp(80)] (finite in bf16); the scaled K
  // and Q are written over the raw tiles and serve the W product and the
  // state pass as well.  Slow path: per-row-block reference points (above).
  // The scaled tiles are bf16 for either I/O type (f16 has no room for
  // exp(80)); what goes to the workspace is converted to the I/O type.
  KTRACE(2);
  if (ok) {
    const float2 gc = *reinterpret_cast<const float2*>(sGb + 4 * 128 + ch);
    const float xc0 = expf(gc.x), xc1 = expf(gc.y);  // the state's per-chunk decay: full accuracy
    if (J == 3) *reinterpret_cast<float2*>(rec + kKWsVec + ch * 4) = make_float2(xc0, xc1);
    if (fast) {
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        const int i = 16 * J + r;
        const uint32_t off = tc::sw128_offset(i, lane >> 2) + (lane & 3) * 4;
        uint32_t* kp = reinterpret_cast<uint32_t*>(smem + kKQ + kb * kKQBlock + off);
        uint32_t* qp = reinterpret_cast<uint32_t*>(smem + kKQ + kb * kKQBlock + 8192 + off);
        const uint32_t kw = *kp, qw = *qp;
        const float k0 = tc::unpack_lo<BF16>(kw), k1 = tc::unpack_hi<BF16>(kw);
        const float q0 = tc::unpack_lo<BF16>(qw), q1 = tc::unpack_hi<BF16>(qw);
        const float x0 = __expf(G0[r]), x1 = __expf(G1[r]);
        const float n0 = k0 * __expf(-G0[r]), n1 = k1 * __expf(-G1[r]);
        *kp = tc::pack2<true>(k0 * x0, k1 * x1);
        *qp = tc::pack2<true>(q0 * x0, q1 * x1);
        *reinterpret_cast<uint32_t*>(smem + oKnF + kb * 8192 + off) = tc::pack2<true>(n0, n1);
        *reinterpret_cast<uint32_t*>(rec + kKWsKd + kb * 8192 + off) = tc::pack2<false>(n0 * xc0, n1 * xc1);
      }
    } else {
      float gbI0[4], gbI1[4];
#pragma unroll
      for (int I = 0; I < 4; ++I) {
        const float2 v = *reinterpret_cast<const float2*>(sGb + I * 128 + ch);
        gbI0[I] = v.x;
        gbI1[I] = v.y;
      }
      float qg0[16], qg1[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        const int i = 16 * J + r;
        const uint32_t off = tc::sw128_offset(i, lane >> 2) + (lane & 3) * 4;
        uint32_t* kp = reinterpret_cast<uint32_t*>(smem + kKQ + kb * kKQBlock + off);
        uint32_t* qp = reinterpret_cast<uint32_t*>(smem + kKQ + kb * kKQBlock + 8192 + off);
        const uint32_t kw = *kp, qw = *qp;
        const float k0 = tc::unpack_lo<BF16>(kw), k1 = tc::unpack_hi<BF16>(kw);
        const float q0 = tc::unpack_lo<BF16>(qw), q1 = tc::unpack_hi<BF16>(qw);
        // every factor an exponential of a non-positive argument (the
        // diagonal block's right factors are clamped and replaced later)
        const float x0 = __expf(G0[r]), x1 = __expf(G1[r]);
        const float ea0 = __expf(G0[r] - gbI0[J]), ea1 = __expf(G1[r] - gbI1[J]);
        const float kd0 = __expf(gc.x - G0[r]), kd1 = __expf(gc.y - G1[r]);
        *kp = tc::pack2<true>(k0 * ea0, k1 * ea1);
        *qp = tc::pack2<true>(q0 * ea0, q1 * ea1);
        *reinterpret_cast<uint32_t*>(smem + kKg + kb * 8192 + off) = tc::pack2<true>(k0 * x0, k1 * x1);
        *reinterpret_cast<uint32_t*>(rec + kKWsKd + kb * 8192 + off) = tc::pack2<false>(k0 * kd0, k1 * kd1);
#pragma unroll
        for (int I = 0; I < 4; ++I)
          if (I >= J)
            *reinterpret_cast<uint32_t*>(smem + kKn + kn_off(I) + kb * kn_blk(I) + off) =
                tc::pack2<true>(k0 * __expf(fminf(gbI0[I] - G0[r], 80.f)),
                                k1 * __expf(fminf(gbI1[I] - G1[r], 80.f)));
        qg0[r] = q0 * x0;
        qg1[r] = q1 * x1;
      }
      // (Q . exp(G))^T rows ch, ch + 1, tokens 16 J .. 16 J + 15: two 16-byte pieces each
#pragma unroll
      for (int h8 = 0; h8 < 2; ++h8) {
        const float* s0 = qg0 + 8 * h8;
        const float* s1 = qg1 + 8 * h8;
        *reinterpret_cast<uint4*>(rec + kKWsQT + tc::sw128_offset(ch, 2 * J + h8)) =
            make_uint4(tc::pack2<BF16>(s0[0], s0[1]), tc::pack2<BF16>(s0[2], s0[3]),
                       tc::pack2<BF16>(s0[4], s0[5]), tc::pack2<BF16>(s0[6], s0[7]));
        *reinterpret_cast<uint4*>(rec + kKWsQT + tc::sw128_offset(ch + 1, 2 * J + h8)) =
            make_uint4(tc::pack2<BF16>(s1[0], s1[1]), tc::pack2<BF16>(s1[2], s1[3]),
                       tc::pack2<BF16>(s1[4], s1[5]), tc::pack2<BF16>(s1[6], s1[7]));
      }
    }
    tc::fence_proxy_async();  // the scaled tiles are MMA operands
  }
  tc::fence_before_sync();
  __syncthreads();
  if (ok && tid == 0) {
    tc::fence_after_sync();
    if (fast) {  // one N = 64 product into the columns of row block 3
      constexpr uint32_t idesc = tc::idesc_f16(128, 64, false, false, true);
#pragma unroll
      for (int s = 0; s < 8; ++s)
        tc::mma(tmem + oTmFast, tc::kmajor_desc(sb + kKQ, kKQBlock, s),
                tc::kmajor_desc(sb + oKnF, 8192, s), idesc, s > 0);
    } else {  // per row block I: [K-rows; Q-rows] x right factors of block I
#pragma unroll
      for (int I = 0; I < 4; ++I) {
        const uint32_t idesc = tc::idesc_f16(128, 16 * (I + 1), false, false, true);
#pragma unroll
        for (int s = 0; s < 8; ++s)
          tc::mma(tmem + 8 * I * (I + 1), tc::kmajor_desc(sb + kKQ, kKQBlock, s),
                  tc::kmajor_desc(sb + kKn + kn_off(I), kn_blk(I), s), idesc, s > 0);
      }
    }
    tc::commit(&bars[1]);
  }
  KTRACE(3);
  if (ok) ok = !named_barrier_or(1, kThreads, (lane == 0) && !mbar_wait_bounded(&bars[1], par));
  KTRACE(4);
  float* sG = reinterpret_cast<float*>(smem + kGs);
  if (ok) {
    tc::fence_after_sync();
    if (!fast) {  // G table for the direct diagonal blocks (the right factors are consumed),
                  // recomputed from the gates so that G need not stay in registers
      uint32_t h0[16], h1[16];
      float F0[16], F1[16], o0, o1;
      load_gates(h0, h1);
      block_scan(h0, h1, F0, F1);
      block_offset(o0, o1);
#pragma unroll
      for (int r = 0; r < 16; ++r)
        *reinterpret_cast<float2*>(sG + (16 * J + r) * kGLd + ch) = make_float2(F0[r] + o0, F1[r] + o1);
    }
  }
  __syncthreads();
  // A -> T: over the consumed right factors (fast path: the scaled K / Q tiles
  // are still needed) or over the K / Q tiles (slow path)
  float* AT = reinterpret_cast<float*>(smem + (fast ? oATF : kAT));
  float* Ms = AT + 64 * kLd;
  const int q4 = warp & 3, hw = warp >> 2;
  const uint32_t lane_q = static_cast<uint32_t>(q4 * 32) << 16;
  if (ok) {
    // ---- A and P rows.  Warp quarter q4 reads TMEM lanes 32 q4 .. (q4 < 2: A
    // rows, else P rows) and the warp pair (w, w + 4) splits the work.
    const bool isA = q4 < 2;
    const int i = 32 * (q4 & 1) + lane;
    const int lim = isA ? i : i + 1;  // A: j < i; P: j <= i
    if (fast) {  // warp half hw: columns 32 hw .. 32 hw + 31
      float r[32];
      tc::tmem_ld16(tmem + lane_q + oTmFast + 32 * hw, *reinterpret_cast<float(*)[16]>(r));
      tc::tmem_ld16(tmem + lane_q + oTmFast + 32 * hw + 16, *reinterpret_cast<float(*)[16]>(r + 16));
      tc::tmem_wait_ld();
      if (isA) {
        const float bi = sBeta[i];
#pragma unroll
        for (int j4 = 0; j4 < 32; j4 += 4) {
          const int j = 32 * hw + j4;
          *reinterpret_cast<float4*>(AT + i * kLd + j) =
              make_float4(j < lim ? bi * r[j4] : 0.f, j + 1 < lim ? bi * r[j4 + 1] : 0.f,
                          j + 2 < lim ? bi * r[j4 + 2] : 0.f, j + 3 < lim ? bi * r[j4 + 3] : 0.f);
        }
      } else {
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = (32 * hw + 8 * c8 + e < lim) ? r[8 * c8 + e] : 0.f;
          tc::sts128(sb + oTu + tc::sw128_offset(i, 4 * hw + c8), tc::pack2<BF16>(v[0], v[1]),
                     tc::pack2<BF16>(v[2], v[3]), tc::pack2<BF16>(v[4], v[5]), tc::pack2<BF16>(v[6], v[7]));
        }
      }
    } else {  // the warp half hw serves the lanes of row block Iw
      const int Iw = 2 * (q4 & 1) + hw;
      float r[64];
#pragma unroll
      for (int cb = 0; cb < 4; ++cb)
        if (cb <= Iw)
          tc::tmem_ld16(tmem + lane_q + 8 * Iw * (Iw + 1) + cb * 16, *reinterpret_cast<float(*)[16]>(r + 16 * cb));
      tc::tmem_wait_ld();
      if ((lane >> 4) == hw) {
        float dg[16];
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) dg[jj] = 0.f;
        if (t0 + i < T) {  // direct diagonal block
          const IO* src = static_cast<const IO*>(isA ? a.k : a.q);
          const IO* krow = static_cast<const IO*>(a.k);
          const int64_t rs = static_cast<int64_t>(a.Hqk) * kD;  // token stride
          const int64_t base = (static_cast<int64_t>(b) * T + t0) * rs + static_cast<int64_t>(hq) * kD;
          const uint32_t* arow = reinterpret_cast<const uint32_t*>(src + base + i * rs);
          const float* Gi = sG + i * kGLd;
          for (int cp = 0; cp < 64; ++cp) {
            const uint32_t aw = __ldg(arow + cp);
            const float a0 = tc::unpack_lo<BF16>(aw), a1 = tc::unpack_hi<BF16>(aw);
            const float2 gi = *reinterpret_cast<const float2*>(Gi + 2 * cp);
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const int j = 16 * Iw + jj;
              if (j < lim && t0 + j < T) {
                const uint32_t kw = __ldg(reinterpret_cast<const uint32_t*>(krow + base + j * rs) + cp);
                const float2 gj = *reinterpret_cast<const float2*>(sG + j * kGLd + 2 * cp);
                dg[jj] += a0 * tc::unpack_lo<BF16>(kw) * __expf(gi.x - gj.x) +
                          a1 * tc::unpack_hi<BF16>(kw) * __expf(gi.y - gj.y);
              }
            }
          }
        }
        auto val = [&](int j) -> float {  // j compile-time after unrolling
          const float v = ((j >> 4) == Iw) ? dg[j & 15] : r[j];
          return j < lim ? v : 0.f;
        };
        if (isA) {
          const float bi = sBeta[i];
#pragma unroll
          for (int j4 = 0; j4 < 64; j4 += 4)
            *reinterpret_cast<float4*>(AT + i * kLd + j4) =
                make_float4(bi * val(j4), bi * val(j4 + 1), bi * val(j4 + 2), bi * val(j4 + 3));
        } else {
#pragma unroll
          for (int c8 = 0; c8 < 8; ++c8)
            tc::sts128(sb + oTu + tc::sw128_offset(i, c8), tc::pack2<BF16>(val(8 * c8), val(8 * c8 + 1)),
                       tc::pack2<BF16>(val(8 * c8 + 2), val(8 * c8 + 3)),
                       tc::pack2<BF16>(val(8 * c8 + 4), val(8 * c8 + 5)),
                       tc::pack2<BF16>(val(8 * c8 + 6), val(8 * c8 + 7)));
        }
      }
    }
    tc::fence_proxy_async();  // the P tile is read by a bulk copy
  }
  __syncthreads();
  KTRACE(5);
  if (ok && tid == 0) {
    bulk_s2g(rec + kKWsP, smem + oTu, 8192);
    bulk_commit();
  }
  if (ok && warp < 4) solve_unit_lower(AT, Ms, warp, lane, 2);
  if (ok && fast && warp >= 4) {
    // meanwhile: (Q . exp(G))^T, MN-major rows d_k, from the scaled Q tile by
    // 8 x 8 transposes written straight to the record; warp w - 4 takes d_k
    // rows 32 (w - 4) .. + 31.  Lane t holds, for transposed block mm, row
    // t / 4 and the column pair 2 (t % 4) of that 8 x 8 block.
    const int w = warp - 4, m = lane >> 3, r8 = lane & 7;
    const uint32_t qsrc = sb + kKQ + 8192;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int kc = w * 4 + j;  // d_k rows 8 kc .. 8 kc + 7
      const uint32_t src = qsrc + (kc >> 3) * kKQBlock;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t v[4];
        tc::ldsm_x4_trans(src + tc::sw128_offset(8 * (4 * hh + m) + r8, kc & 7), v);
#pragma unroll
        for (int mm = 0; mm < 4; ++mm) {
          const uint32_t x = BF16 ? v[mm] : tc::pack2<false>(tc::unpack_lo<true>(v[mm]), tc::unpack_hi<true>(v[mm]));
          *reinterpret_cast<uint32_t*>(rec + kKWsQT + tc::sw128_offset(8 * kc + (lane >> 2), 4 * hh + mm) +
                                       4 * (lane & 3)) = x;
        }
      }
    }
  }
  if (ok && tid == 0) bulk_wait_read();  // the P staging tile may be overwritten
  __syncthreads();
  if (ok && warp < 4) {
    // T_u = T diag(beta): rows 16 w .. 16 w + 15; lane l the 16-byte chunk l % 8
    // of rows 16 w + l / 8 + 4 s (four whole rows per store instruction), to
    // the record (I/O type) and to the W-product operand tile (bf16)
    const int c8 = lane & 7;
    const float4 b0 = *reinterpret_cast<const float4*>(sBeta + 8 * c8);
    const float4 b1 = *reinterpret_cast<const float4*>(sBeta + 8 * c8 + 4);
    const float bj[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    float4 ua[4], ub4[4];  // loads first (the stores below would order them)
#pragma unroll
    for (int s4 = 0; s4 < 4; ++s4) {
      const int i = 16 * warp + (lane >> 3) + 4 * s4;
      ua[s4] = *reinterpret_cast<const float4*>(AT + i * kLd + 8 * c8);
      ub4[s4] = *reinterpret_cast<const float4*>(AT + i * kLd + 8 * c8 + 4);
    }
#pragma unroll
    for (int s4 = 0; s4 < 4; ++s4) {
      const int i = 16 * warp + (lane >> 3) + 4 * s4;
      const float4 u0 = ua[s4], u1 = ub4[s4];
      const float tv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
      uint32_t uu[4], ub[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j0 = 8 * c8 + 2 * e;
        const float v0 = (j0 <= i) ? tv[2 * e] * bj[2 * e] : 0.f;
        const float v1 = (j0 + 1 <= i) ? tv[2 * e + 1] * bj[2 * e + 1] : 0.f;
        uu[e] = tc::pack2<BF16>(v0, v1);
        ub[e] = BF16 ? uu[e] : tc::pack2<true>(v0, v1);
      }
      const uint32_t off = tc::sw128_offset(i, c8);
      *reinterpret_cast<uint4*>(rec + kKWsTu + off) = make_uint4(uu[0], uu[1], uu[2], uu[3]);
      tc::sts128(sb + oTu + off, ub[0], ub[1], ub[2], ub[3]);
    }
    tc::fence_proxy_async();
  }
  tc::fence_before_sync();
  __syncthreads();
  KTRACE(7);
  if (ok && tid == 0) {  // W^T = (K . exp(G))^T T_u^T
    tc::fence_after_sync();
    constexpr uint32_t kIdW = tc::idesc_f16(128, 64, true, false, true);
#pragma unroll
    for (int s = 0; s < 4; ++s)
      tc::mma(tmem + oTmW, fast ? tc::mnmajor_desc(sb + kKQ, kKQBlock, s) : tc::mnmajor_desc(sb + kKg, 8192, s),
              tc::kmajor_desc(sb + oTu, 0, s), kIdW, s > 0);
    tc::commit(&bars[2]);
  }
  if (ok) ok = !named_barrier_or(1, kThreads, (lane == 0) && !mbar_wait_bounded(&bars[2], par));
  if (ok) {  // W^T rows d_k = 32 q4 + lane, tokens 32 hw .. 32 hw + 31, MN-major
    tc::fence_after_sync();
    const int k = q4 * 32 + lane;
    float r[32];
    tc::tmem_ld16(tmem + lane_q + oTmW + hw * 32, *reinterpret_cast<float(*)[16]>(r));
    tc::tmem_ld16(tmem + lane_q + oTmW + hw * 32 + 16, *reinterpret_cast<float(*)[16]>(r + 16));
    tc::tmem_wait_ld();
    store_row16_global<BF16>(rec + kKWsWT, k, hw * 4, r);
    store_row16_global<BF16>(rec + kKWsWT, k, hw * 4 + 2, r + 16);
  }
  KTRACE(8);
  if (!ok && tid == 0) report(a.status, GDN_DEVERR_MMA_TIMEOUT);
  if (tid == 0) bulk_wait_all();  // the P tile has left shared memory
  tc::fence_before_sync();
  __syncthreads();
  KTRACE(9);
  tc::fence_proxy_async();  // generic writes before the next unit's TMA into the same bytes
  return true;
}

// Fast-path kernel: one CTA per unit, three per SM.  Units outside the fast
// path's range go to a device list for kda_intra_slow.
template <bool BF16>
__global__ void __launch_bounds__(kintra::kThreads, 3)
    kda_intra_fast(const Params p, const __grid_constant__ CUtensorMap map_q,
                   const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_g) {
  using namespace kintra;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kFoBars);  // [0] TMA, [1] A/P MMA, [2] W MMA
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 3);
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x < 32) tc::tmem_alloc(tmem_holder, kFoTmCols);
  if (threadIdx.x == 0) {
    for (int i = 0; i < 3; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  const int unit = static_cast<int>(blockIdx.x);
  if (!kda_unit<BF16, true>(p, map_q, map_k, map_g, unit, 0, smem, bars, tmem) && threadIdx.x == 0)
    p.slow_list[atomicAdd(p.slow_count, 1u)] = unit;
  tc::fence_before_sync();
  __syncthreads();
  if (threadIdx.x < 32) tc::tmem_dealloc(tmem, kFoTmCols);
}

// Slow-path kernel: a persistent grid over the units kda_intra_fast deferred
// (usually none; it then exits at once).
template <bool BF16>
__global__ void __launch_bounds__(kintra::kThreads, 2)
    kda_intra_slow(const Params p, const __grid_constant__ CUtensorMap map_q,
                   const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_g) {
  using namespace kintra;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBars);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 3);
  pdl_wait();  // the list is complete
  const int n = static_cast<int>(*reinterpret_cast<volatile uint32_t*>(p.slow_count));
  if (static_cast<int>(blockIdx.x) >= n) {
    pdl_launch_dependents();
    return;
  }
  if (threadIdx.x < 32) tc::tmem_alloc(tmem_holder, kTmCols);
  if (threadIdx.x == 0) {
    for (int i = 0; i < 3; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  uint32_t par = 0;
  for (int i = static_cast<int>(blockIdx.x); i < n; i += static_cast<int>(gridDim.x), par ^= 1u)
    kda_unit<BF16, false>(p, map_q, map_k, map_g, p.slow_list[i], par, smem, bars, tmem);
  pdl_launch_dependents();
  tc::fence_before_sync();
  __syncthreads();
  if (threadIdx.x < 32) tc::tmem_dealloc(tmem, kTmCols);
}

size_t workspace_bytes(const gdn_prefill_args_t& a) {
  const size_t nchunks = (static_cast<size_t>(a.T) + kC - 1) / kC;
  return static_cast<size_t>(a.B) * a.Hv * nchunks * kWsUnit;
}

template <bool BF16>
int launch(const gdn_prefill_args_t& a, cudaStream_t stream) {
  static std::atomic<uint64_t> attr_intra{0}, attr_state{0};
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  if (static_cast<int>(state::kSmemAlloc) > di.smem_optin) return GDN_ERR_SHAPE;
  auto k1 = intra_kernel<BF16>;
  auto k2 = state_kernel<BF16, false>;
  if ((rc = ensure_smem_attr(k1, intra::kSmemAlloc, attr_intra))) return rc;
  if ((rc = ensure_smem_attr(k2, state::kSmemAlloc, attr_state))) return rc;
  const CUtensorMapDataType dt = BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap mq, mk, mv;
  const uint32_t box[4] = {64, 1, kC, 1};
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(a.dk), static_cast<uint64_t>(a.Hqk),
                              static_cast<uint64_t>(a.T), static_cast<uint64_t>(a.B)};
    const uint64_t str[3] = {static_cast<uint64_t>(a.dk) * 2, static_cast<uint64_t>(a.Hqk) * a.dk * 2,
                             static_cast<uint64_t>(a.T) * a.Hqk * a.dk * 2};
    if ((rc = tensor_map(&mq, dt, 4, a.q, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
    if ((rc = tensor_map(&mk, dt, 4, a.k, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  }
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(a.dv), static_cast<uint64_t>(a.Hv),
                              static_cast<uint64_t>(a.T), static_cast<uint64_t>(a.B)};
    const uint64_t str[3] = {static_cast<uint64_t>(a.dv) * 2, static_cast<uint64_t>(a.Hv) * a.dv * 2,
                             static_cast<uint64_t>(a.T) * a.Hv * a.dv * 2};
    if ((rc = tensor_map(&mv, dt, 4, a.v, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  }
  Params p;
  p.a = a;
  p.nchunks = (a.T + kC - 1) / kC;
  p.group = a.Hv / a.Hqk;
  p.ws = static_cast<unsigned char*>(a.workspace);
  p.slow_count = nullptr;
  p.slow_list = nullptr;
  const unsigned n1 = static_cast<unsigned>(a.B * a.Hqk * p.nchunks);
  k1<<<n1, intra::kThreads, intra::kSmemAlloc, stream>>>(p, mq, mk);
  if (cudaGetLastError() != cudaSuccess) return GDN_ERR_LAUNCH;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a.B * a.Hv));
  cfg.blockDim = dim3(state::kThreads);
  cfg.dynamicSmemBytes = state::kSmemAlloc;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, k2, p, mq, mk, mv) != cudaSuccess) {
    (void)cudaGetLastError();
    return GDN_ERR_LAUNCH;
  }
  return GDN_OK;
}

// KDA workspace: the records, then the count (16 bytes) and the list of
// units deferred to the slow-path kernel.
size_t kda_records_bytes(const gdn_prefill_args_t& a) {
  const size_t nchunks = (static_cast<size_t>(a.T) + kC - 1) / kC;
  return static_cast<size_t>(a.B) * a.Hv * nchunks * kKWsUnit;
}
size_t kda_workspace_bytes(const gdn_prefill_args_t& a) {
  const size_t units = kda_records_bytes(a) / kKWsUnit;
  return kda_records_bytes(a) + 16 + ((units * 4 + 15) & ~size_t(15));
}

// KDA chunked prefill: the deferred-unit count cleared, kda_intra_fast, then
// kda_intra_slow and state_kernel<., true> as programmatic dependents.
// Arguments validated by the caller.
template <bool BF16>
int launch_kda(const gdn_prefill_args_t& a, cudaStream_t stream) {
  static std::atomic<uint64_t> attr_fast{0}, attr_slow{0}, attr_state{0};
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  if (static_cast<int>(state::kSmemAlloc) > di.smem_optin) return GDN_ERR_SHAPE;
  auto k1 = kda_intra_fast<BF16>;
  auto k1s = kda_intra_slow<BF16>;
  auto k2 = state_kernel<BF16, true>;
  if ((rc = ensure_smem_attr(k1, kintra::kFoSmemAlloc, attr_fast))) return rc;
  if ((rc = ensure_smem_attr(k1s, kintra::kSmemAlloc, attr_slow))) return rc;
  if ((rc = ensure_smem_attr(k2, state::kSmemAlloc, attr_state))) return rc;
  const CUtensorMapDataType dt = BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap mq, mk, mv;
  const uint32_t box[4] = {64, 1, kC, 1};
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(a.dk), static_cast<uint64_t>(a.Hqk),
                              static_cast<uint64_t>(a.T), static_cast<uint64_t>(a.B)};
    const uint64_t str[3] = {static_cast<uint64_t>(a.dk) * 2, static_cast<uint64_t>(a.Hqk) * a.dk * 2,
                             static_cast<uint64_t>(a.T) * a.Hqk * a.dk * 2};
    if ((rc = tensor_map(&mq, dt, 4, a.q, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
    if ((rc = tensor_map(&mk, dt, 4, a.k, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  }
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(a.dv), static_cast<uint64_t>(a.Hv),
                              static_cast<uint64_t>(a.T), static_cast<uint64_t>(a.B)};
    const uint64_t str[3] = {static_cast<uint64_t>(a.dv) * 2, static_cast<uint64_t>(a.Hv) * a.dv * 2,
                             static_cast<uint64_t>(a.T) * a.Hv * a.dv * 2};
    if ((rc = tensor_map(&mv, dt, 4, a.v, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  }
  CUtensorMap mg;  // per-channel gates [B, T, Hv, d_k], one chunk x all channels per box
  {
    const uint64_t es = a.g_dtype == GDN_DT_F32 ? 4 : 2;
    const CUtensorMapDataType gdt = a.g_dtype == GDN_DT_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                    : a.g_dtype == GDN_DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint64_t dims[4] = {static_cast<uint64_t>(a.dk), static_cast<uint64_t>(a.Hv),
                              static_cast<uint64_t>(a.T), static_cast<uint64_t>(a.B)};
    const uint64_t str[3] = {a.dk * es, static_cast<uint64_t>(a.Hv) * a.dk * es,
                             static_cast<uint64_t>(a.T) * a.Hv * a.dk * es};
    const uint32_t gbox[4] = {static_cast<uint32_t>(kD), 1, kC, 1};
    if ((rc = tensor_map(&mg, gdt, 4, a.g, dims, str, gbox, CU_TENSOR_MAP_SWIZZLE_NONE))) return rc;
  }
  Params p;
  p.a = a;
  p.nchunks = (a.T + kC - 1) / kC;
  p.group = a.Hv / a.Hqk;
  p.ws = static_cast<unsigned char*>(a.workspace);
  p.slow_count = reinterpret_cast<uint32_t*>(p.ws + kda_records_bytes(a));
  p.slow_list = reinterpret_cast<int32_t*>(p.ws + kda_records_bytes(a) + 16);
  const unsigned n1 = static_cast<unsigned>(a.B * a.Hv * p.nchunks);
  if (cudaMemsetAsync(p.slow_count, 0, sizeof(uint32_t), stream) != cudaSuccess) return GDN_ERR_LAUNCH;
  k1<<<n1, kintra::kThreads, kintra::kFoSmemAlloc, stream>>>(p, mq, mk, mg);
  if (cudaGetLastError() != cudaSuccess) return GDN_ERR_LAUNCH;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cs = {};
  cs.gridDim = dim3(std::min(n1, static_cast<unsigned>(2 * di.sm_count)));
  cs.blockDim = dim3(kintra::kThreads);
  cs.dynamicSmemBytes = kintra::kSmemAlloc;
  cs.stream = stream;
  cs.attrs = attr;
  cs.numAttrs = 1;
  if (cudaLaunchKernelEx(&cs, k1s, p, mq, mk, mg) != cudaSuccess) {
    (void)cudaGetLastError();
    return GDN_ERR_LAUNCH;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a.B * a.Hv));
  cfg.blockDim = dim3(state::kThreads);
  cfg.dynamicSmemBytes = state::kSmemAlloc;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, k2, p, mq, mk, mv) != cudaSuccess) {
    (void)cudaGetLastError();
    return GDN_ERR_LAUNCH;
  }
  return GDN_OK;
}

int validate(const gdn_prefill_args_t* a) {
  if (!a) return GDN_ERR_NULL;
  if (!a->q || !a->k || !a->v || !a->g || !a->beta || !a->final_state || !a->o) return GDN_ERR_NULL;
  if (a->B < 1 || a->T < 1 || a->Hqk < 1 || a->Hv < 1 || a->Hv % a->Hqk) return GDN_ERR_SHAPE;
  if (a->dk != kD || a->dv != kD || a->chunk != kC) return GDN_ERR_SHAPE;
  const int64_t nchunks = (static_cast<int64_t>(a->T) + kC - 1) / kC;
  if (static_cast<int64_t>(a->B) * a->Hv > 0x7FFFFFFF ||
      static_cast<int64_t>(a->B) * a->Hqk * nchunks > 0x7FFFFFFF)
    return GDN_ERR_SHAPE;
  if (a->io_dtype != GDN_DT_BF16 && a->io_dtype != GDN_DT_F16) return GDN_ERR_DTYPE;
  if (!dtype_valid(a->g_dtype) || !dtype_valid(a->beta_dtype)) return GDN_ERR_DTYPE;
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->o) ||
      !aligned16(a->final_state) || (a->initial_state && !aligned16(a->initial_state)))
    return GDN_ERR_ALIGN;
  if (!a->workspace || a->workspace_bytes < workspace_bytes(*a)) return GDN_ERR_WORKSPACE;
  if (!aligned16(a->workspace)) return GDN_ERR_ALIGN;
  return GDN_OK;
}

// The chunked KDA path: d_k = d_v = 128 with a workspace (gdn_prefill
// shapes otherwise); called by kda_prefill_launch after its own checks.
int kda_chunked_launch(const gdn_prefill_args_t& a, cudaStream_t stream) {
  if (a.dk != kD || a.dv != kD) return GDN_ERR_SHAPE;
  const int64_t nchunks = (static_cast<int64_t>(a.T) + kC - 1) / kC;
  if (static_cast<int64_t>(a.B) * a.Hv * nchunks > 0x7FFFFFFF) return GDN_ERR_SHAPE;
  if (!a.workspace || a.workspace_bytes < kda_workspace_bytes(a)) return GDN_ERR_WORKSPACE;
  if (!aligned16(a.workspace) || !aligned16(a.final_state) ||
      (a.initial_state && !aligned16(a.initial_state)))
    return GDN_ERR_ALIGN;
  return a.io_dtype == GDN_DT_BF16 ? launch_kda<true>(a, stream) : launch_kda<false>(a, stream);
}

}  // namespace prefill
}  // namespace gdn

extern "C" size_t kda_prefill_workspace_size(const gdn_prefill_args_t* args) {
  if (!args || args->B < 1 || args->T < 1 || args->Hv < 1) return 0;
  if (args->dk != gdn::prefill::kD || args->dv != gdn::prefill::kD) return 0;  // recurrent form
  return gdn::prefill::kda_workspace_bytes(*args);
}

#ifdef GDN_PREFILL_TRACE
extern "C" int gdn_prefill_cta_read(unsigned long long* host) {
  return cudaMemcpyFromSymbol(host, gdn::prefill::g_cta, sizeof(gdn::prefill::g_cta)) == cudaSuccess ? 0 : 1;
}
extern "C" int gdn_prefill_trace1_read(unsigned long long* host) {
  return cudaMemcpyFromSymbol(host, gdn::prefill::g_trace1, sizeof(gdn::prefill::g_trace1)) ==
                 cudaSuccess
             ? 0
             : 1;
}
extern "C" int kda_intra_trace_read(unsigned long long* host) {
  return cudaMemcpyFromSymbol(host, gdn::prefill::g_ktrace, sizeof(gdn::prefill::g_ktrace)) == cudaSuccess ? 0 : 1;
}
extern "C" int gdn_prefill_trace_read(unsigned long long* host) {
  return cudaMemcpyFromSymbol(host, gdn::prefill::g_trace, sizeof(gdn::prefill::g_trace)) ==
                 cudaSuccess
             ? 0
             : 1;
}
#endif

extern "C" size_t gdn_prefill_workspace_size(const gdn_prefill_args_t* args) {
  if (!args || args->B < 1 || args->T < 1 || args->Hv < 1) return 0;
  return gdn::prefill::workspace_bytes(*args);
}

extern "C" int gdn_prefill_launch(const gdn_prefill_args_t* args, gdn_stream_t stream) {
  int rc = gdn::prefill::validate(args);
  if (rc) return rc;
  gdn::DeviceInfo di;
  if ((rc = gdn::device_info(&di))) return rc;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  return args->io_dtype == GDN_DT_BF16 ? gdn::prefill::launch<true>(*args, s)
                                       : gdn::prefill::launch<false>(*args, s);
}

// ------------------------------------------------------------------------
// gdn_prefill_launch_noalloc: the same two kernels, with their workspace in a
// fixed device array instead of caller-provided memory, for callers that
// cannot allocate device memory themselves (see include/gdn_b200.h).
// The array is a module global: every GPU that loads this library holds
// GDN_PREFILL_NOALLOC_SCRATCH_BYTES of it until the process exits, and all
// calls on a device share it.  Host code must not pass the symbol itself to a
// kernel (on the host it names a host-side stand-in); its device address is
// looked up once per device with cudaGetSymbolAddress, with that device
// current, on the first call there.
namespace {

static __device__ __align__(256) unsigned char g_prefill_noalloc_scratch[GDN_PREFILL_NOALLOC_SCRATCH_BYTES];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};  // device address of the array, per device ordinal

int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return GDN_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_prefill_noalloc_scratch) != cudaSuccess || !p) return GDN_ERR_DEVICE;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return GDN_OK;
}

}  // namespace

static_assert(gdn::prefill::kWsUnit == GDN_PREFILL_WS_RECORD_BYTES, "record size in the header");

extern "C" int gdn_prefill_launch_noalloc(const gdn_prefill_args_t* args, gdn_stream_t stream) {
  if (!args) return GDN_ERR_NULL;
  if (args->B < 1 || args->T < 1 || args->Hv < 1) return GDN_ERR_SHAPE;
  gdn_prefill_args_t a = *args;
  // One record per (sequence, value head, 64-token chunk); nothing in the
  // scratch has to start at zero: the first kernel writes every record the
  // second one reads, in stream order.
  if (gdn::prefill::workspace_bytes(a) > GDN_PREFILL_NOALLOC_SCRATCH_BYTES) return GDN_ERR_WORKSPACE;
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  a.workspace = scratch;
  a.workspace_bytes = GDN_PREFILL_NOALLOC_SCRATCH_BYTES;
  return gdn_prefill_launch(&a, stream);
}
