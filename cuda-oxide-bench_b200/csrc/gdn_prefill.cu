// gdn_prefill.cu — GDN chunked prefill on the sm_100a tensor cores (tcgen05).
//
// The reference defines prefill only as T applications of its decode
// recurrence (pytorch_reference_gdn.py:38-91; chunking is described, not
// implemented, in analysis/wave15-attention-research/MECHANISMS.md:398-445).
// This kernel computes the same result chunk by chunk (chunk C = 64 tokens).
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
// Every product is a tcgen05.mma with M = 128, written transposed so the 128
// TMEM lanes index d_v (or d_k): [K;Q] K^T, W^T = K^T T_w^T, U^T = V^T T_u^T,
// V'^T = U^T - S^T W^T (accumulated with a negated A onto U), Z^T = S^T Q^T,
// O_intra^T = V'^T P^T, dS^T = V''^T K.  Operands are bf16 (f16) in
// 128B-swizzled shared memory (TMA fills K/Q/V; one tile serves as K-major and
// MN-major operand), except S^T, which lives in TMEM as bf16 and is read as
// the A operand.  Accumulators use all 512 TMEM columns; the fp32 master state
// lives in registers of the state warps.
// Precision: the decayed V'' = diag(exp(G_C - G_j)) V' that updates the state
// is split into bf16 hi + lo halves (two MMAs), and K enters the state update
// unscaled, so the state accumulates with ~16 mantissa bits per term.
//
// One CTA per (batch, value head), 16 warps in two roles that run
// concurrently, one chunk apart:
//   intra (warps 0-7):   KQ MMA, A and P rows, T = (I+A)^-1, W/U MMAs, W^T tile
//                        for chunk c+1 ...
//   state (warps 8-15):  ... while the state chain of chunk c runs: V' = U - W S,
//                        V'/V'' tiles, O_intra/dS MMAs, state update, outputs.
// K/Q/V are double-buffered; the state warps' MMA thread refills a slot with
// chunk c+2 by TMA as soon as chunk c's last MMA on it has completed.
// Hand-offs use mbarriers (TMA completion, tcgen05.commit, group arrivals); every
// wait is bounded and each group agrees on an abort before leaving its loop.
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "ptx.cuh"
#include "tc.cuh"

namespace gdn {
namespace prefill {

#ifdef GDN_PREFILL_TRACE
// Phase timestamps of CTA 0 (profiling builds only): [chunk][phase].
__device__ unsigned long long g_trace[64 * 16];
#define TRACE(c, ph)                                                                           \
  do {                                                                                         \
    if (blockIdx.x == 0 && (c) < 64 && (threadIdx.x == 0 || threadIdx.x == kIntraThreads))              \
      g_trace[(c) * 16 + (ph)] = global_timer_ns();                                            \
  } while (0)
#else
#define TRACE(c, ph) \
  do {               \
  } while (0)
#endif

constexpr int kC = 64;     // chunk length
constexpr int kD = 128;    // d_k = d_v
constexpr int kIntraThreads = 256;
constexpr int kStateThreads = 256;
constexpr int kThreads = kIntraThreads + kStateThreads;
constexpr int kBarIntra = 1, kBarState = 2;  // named barrier ids

// shared-memory map (byte offsets from a 1024-aligned base)
constexpr uint32_t kKQ = 0;            // 2 slots x [K | Q] tile: 2 d_k blocks x (K 8 KB + Q 8 KB)
constexpr uint32_t kKQSlot = 32768;
constexpr uint32_t kKQBlock = 16384;
constexpr uint32_t kV = 65536;         // 2 slots x V tile: 2 d_v blocks x 8 KB
constexpr uint32_t kVSlot = 16384;
constexpr uint32_t kVBlock = 8192;
constexpr uint32_t kTw = 98304;        // T diag(beta gamma), K-major rows i   (8 KB)
constexpr uint32_t kTu = 106496;       // T diag(beta), K-major rows i          (8 KB)
constexpr uint32_t kP = 114688;        // 2 slots x causal decayed QK^T        (8 KB each)
constexpr uint32_t kPSlot = 8192;
constexpr uint32_t kWT = 131072;       // W^T, MN-major rows d_k               (16 KB)
constexpr uint32_t kVP = 147456;       // V'^T, K-major rows d_v               (16 KB)
constexpr uint32_t kVH = 163840;       // V''^T hi                             (16 KB)
constexpr uint32_t kVL = 180224;       // V''^T lo                             (16 KB)
constexpr int kLd = 68;                // fp32 row stride of the solver matrices
constexpr uint32_t kAT = 196608;       // A, overwritten in place by T: [64][68] fp32
constexpr uint32_t kMs = kTw;          // solver scratch [32][68] fp32 (aliases T_w/T_u,
                                       // which are written only after the solve)
constexpr uint32_t kVec = kAT + 64 * kLd * 4;  // 3 slots x {G, gamma, beta, decay} x 64 fp32
constexpr int kVecSlot = 4 * 64;               // floats per slot
constexpr uint32_t kBars = kVec + 3 * kVecSlot * 4;
constexpr uint32_t kSmemBytes = kBars + 256;
constexpr uint32_t kSmemAlloc = kSmemBytes + 1024;  // + alignment slack
static_assert(32 * kLd * 4 <= 2 * 8192, "solver scratch overflows its alias");

// TMEM columns
constexpr uint32_t kTmST = 0;    // S^T bf16, packed pairs: 64 columns
constexpr uint32_t kTmKQ = 64;   // [K;Q]K^T, then reused for W^T
constexpr uint32_t kTmU = 128;   // 2 slots x U^T / V'^T
constexpr uint32_t kTmZ = 256, kTmOI = 320, kTmDS = 384, kTmCols = 512;

// mbarrier indices
enum {
  kBarKQV = 0,        // [2] TMA of a K/Q/V slot landed
  kBarIMma = 2,       // intra MMA completion
  kBarReady = 3,      // [2] intra -> state: W^T tile, U, P, gates of a chunk ready
  kBarX = 5,          // V' = U - W S done (W^T tile free)
  kBarZ = 6,          // Z done
  kBarS2 = 7,         // O_intra and dS done
  kBarSlotFree = 8,   // [2] a K/Q/V, U and P slot may be refilled
  kNumBars = 10,
};

struct Params {
  gdn_prefill_args_t a;
  int32_t nchunks;
  int32_t group;
};

template <bool BF16>
__device__ __forceinline__ void store_row16(uint32_t tile, int row, int chunk0, const float* v) {
  tc::sts128(tile + tc::sw128_offset(row, chunk0), tc::pack2<BF16>(v[0], v[1]),
             tc::pack2<BF16>(v[2], v[3]), tc::pack2<BF16>(v[4], v[5]), tc::pack2<BF16>(v[6], v[7]));
  tc::sts128(tile + tc::sw128_offset(row, chunk0 + 1), tc::pack2<BF16>(v[8], v[9]),
             tc::pack2<BF16>(v[10], v[11]), tc::pack2<BF16>(v[12], v[13]),
             tc::pack2<BF16>(v[14], v[15]));
}

// Bounded wait polled by lane 0 of each warp (the other lanes sleep in the
// barrier instead of competing for issue slots), then a group-wide vote: the
// group leaves together if any warp timed out (no thread is stranded at a
// barrier).  The barrier also orders the waiters' later reads after the phase.
__device__ __forceinline__ bool group_wait(uint64_t* bar, uint32_t parity, int bar_id, int count) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait_bounded(bar, parity);
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

// acc (16 x 16, two m16n8 fragments) += X (16 x 16 block at x, stride kLd) * Y (16 x 16 at y).
__device__ __forceinline__ void block_mma(float (&acc)[2][4], const float* x, const float* y, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int ks = 0; ks < 2; ++ks) {
    uint32_t af[4];
    af[0] = __float_as_uint(x[g * kLd + ks * 8 + t]);
    af[1] = __float_as_uint(x[(g + 8) * kLd + ks * 8 + t]);
    af[2] = __float_as_uint(x[g * kLd + ks * 8 + t + 4]);
    af[3] = __float_as_uint(x[(g + 8) * kLd + ks * 8 + t + 4]);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      uint32_t bf[2];
      bf[0] = __float_as_uint(y[(ks * 8 + t) * kLd + nt * 8 + g]);
      bf[1] = __float_as_uint(y[(ks * 8 + t + 4) * kLd + nt * 8 + g]);
      mma_tf32(acc[nt], af, bf);
    }
  }
}

__device__ __forceinline__ void block_store(float* z, const float (&acc)[2][4], float sign, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    *reinterpret_cast<float2*>(z + g * kLd + nt * 8 + 2 * t) = make_float2(sign * acc[nt][0], sign * acc[nt][1]);
    *reinterpret_cast<float2*>(z + (g + 8) * kLd + nt * 8 + 2 * t) =
        make_float2(sign * acc[nt][2], sign * acc[nt][3]);
  }
}

// In place: AT holds strictly-lower A (64 x 64 fp32, stride kLd, zeros on and
// above the diagonal) and is overwritten with T = (I + A)^-1.  Run by the
// intra warps (warps 0-3 compute; the others only join the group barriers).  Steps: the four 16 x 16 diagonal blocks D_r by
// forward substitution (one warp each, one lane per column, fp32); T_10 =
// -D_1 A_10 D_0 and T_32 = -D_3 A_32 D_2; then the lower-left quadrant
// -T_bot A_bl T_top through Y = A_bl T_top (TF32 warp MMAs).  Each block of A is last read
// before the block of T that replaces it is written.
__device__ __forceinline__ void solve_unit_lower(float* AT, float* M, int warp, int lane) {
  if (warp < 4) {
    const int bb = warp * 16, c = lane & 15;
    float t[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) t[i] = (i == c) ? 1.f : 0.f;
#pragma unroll
    for (int i = 1; i < 16; ++i) {
      const float* row = AT + (bb + i) * kLd + bb;
      float acc = 0.f;
#pragma unroll
      for (int j4 = 0; j4 < i; j4 += 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(row + j4);
        acc = fmaf(a4.x, t[j4], acc);
        if (j4 + 1 < i) acc = fmaf(a4.y, t[j4 + 1], acc);
        if (j4 + 2 < i) acc = fmaf(a4.z, t[j4 + 2], acc);
        if (j4 + 3 < i) acc = fmaf(a4.w, t[j4 + 3], acc);
      }
      t[i] -= acc;
    }
    __syncwarp();
    if (lane < 16) {
#pragma unroll
      for (int i = 0; i < 16; ++i) AT[(bb + i) * kLd + bb + c] = t[i];
    }
  }
  tc::group_sync(kBarIntra, kIntraThreads);
  if (warp < 2) {  // T_10 (warp 0) and T_32 (warp 1)
    const int c = warp * 2, r = c + 1;
    float* X = M + warp * 16 * kLd;
    float acc[2][4] = {};
    block_mma(acc, AT + 16 * r * kLd + 16 * c, AT + 16 * c * kLd + 16 * c, lane);
    block_store(X, acc, 1.f, lane);
    __syncwarp();
    float acc2[2][4] = {};
    block_mma(acc2, AT + 16 * r * kLd + 16 * r, X, lane);
    block_store(AT + 16 * r * kLd + 16 * c, acc2, -1.f, lane);
  }
  tc::group_sync(kBarIntra, kIntraThreads);
  if (warp < 4) {  // Y_rc = sum_k A_rk T_kc over the top blocks, warp (r-2)*2 + c
    const int r = 2 + (warp >> 1), c = warp & 1;
    float acc[2][4] = {};
    if (c == 0) {
      block_mma(acc, AT + 16 * r * kLd + 0, AT + 0, lane);                      // A_r0 D_0
      block_mma(acc, AT + 16 * r * kLd + 16, AT + 16 * kLd + 0, lane);          // A_r1 T_10
    } else {
      block_mma(acc, AT + 16 * r * kLd + 16, AT + 16 * kLd + 16, lane);         // A_r1 D_1
    }
    block_store(M + (r - 2) * 16 * kLd + 16 * c, acc, 1.f, lane);
  }
  tc::group_sync(kBarIntra, kIntraThreads);
  if (warp < 4) {
    const int r = 2 + (warp >> 1), c = warp & 1;
    float acc[2][4] = {};
    if (r == 2) {
      block_mma(acc, AT + 32 * kLd + 32, M + 16 * c, lane);                     // D_2 Y_2c
    } else {
      block_mma(acc, AT + 48 * kLd + 32, M + 16 * c, lane);                     // T_32 Y_2c
      block_mma(acc, AT + 48 * kLd + 48, M + 16 * kLd + 16 * c, lane);          // D_3 Y_3c
    }
    block_store(AT + 16 * r * kLd + 16 * c, acc, -1.f, lane);
  }
  tc::group_sync(kBarIntra, kIntraThreads);
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack_bits(float lo, float hi) {
  return tc::pack2<BF16>(lo, hi);
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const Params p, const __grid_constant__ CUtensorMap map_q,
                   const __grid_constant__ CUtensorMap map_k,
                   const __grid_constant__ CUtensorMap map_v) {
  using IO = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  float* vec = reinterpret_cast<float*>(smem + kVec);  // [slot][G | gamma | beta][64]
  float* AT = reinterpret_cast<float*>(smem + kAT);
  float* Ms = reinterpret_cast<float*>(smem + kMs);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBars);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + kNumBars + 1);

  const gdn_prefill_args_t& a = p.a;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x;
  const int b = bh / a.Hv, h = bh % a.Hv, hq = h / p.group;
  const int T = a.T;
  const int nchunks = p.nchunks;

  if (warp == 0) tc::tmem_alloc(tmem_holder, kTmCols);
  if (tid == 0) {
    mbar_init(&bars[kBarKQV], 1);
    mbar_init(&bars[kBarKQV + 1], 1);
    mbar_init(&bars[kBarIMma], 1);
    mbar_init(&bars[kBarReady], kIntraThreads);
    mbar_init(&bars[kBarReady + 1], kIntraThreads);
    mbar_init(&bars[kBarX], 1);
    mbar_init(&bars[kBarZ], 1);
    mbar_init(&bars[kBarS2], 1);
    mbar_init(&bars[kBarSlotFree], 1);
    mbar_init(&bars[kBarSlotFree + 1], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
  constexpr uint32_t kIdKQ = tc::idesc_f16(128, 64, false, false, BF16);
  constexpr uint32_t kIdW = tc::idesc_f16(128, 64, true, false, BF16);
  constexpr uint32_t kIdXneg = tc::idesc_f16(128, 64, false, true, BF16, true);
  constexpr uint32_t kIdDS = tc::idesc_f16(128, 128, false, true, BF16);

  auto issue_tma = [&](int n) {  // K, Q, V of chunk n into slot n & 1
    const int slot = n & 1;
    uint64_t* bar = &bars[kBarKQV + slot];
    mbar_arrive_expect_tx(bar, 6 * 8192);
    const int t0 = n * kC;
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
      unsigned char* kq = smem + kKQ + slot * kKQSlot + blk * kKQBlock;
      tc::tma_load_4d(kq, &map_k, blk * 64, hq, t0, b, bar);
      tc::tma_load_4d(kq + 8192, &map_q, blk * 64, hq, t0, b, bar);
      tc::tma_load_4d(smem + kV + slot * kVSlot + blk * kVBlock, &map_v, blk * 64, h, t0, b, bar);
    }
  };
  if (tid == kIntraThreads) {
    issue_tma(0);
    if (nchunks > 1) issue_tma(1);
  }

  if (warp < kIntraThreads / 32) {
    // ================================================================ intra
    asm volatile("setmaxnreg.dec.sync.aligned.u32 88;" ::: "memory");
    const int it = tid;  // 0..255
    const int quarter = warp & 3, ih = warp >> 2;
    float g_next = 0.f, b_next = 0.f;
    auto load_gates = [&](int chunk) {
      const int t = chunk * kC + it;
      g_next = 0.f;
      b_next = 0.f;
      if (it < kC && t < T) {
        const int64_t gi = (static_cast<int64_t>(b) * T + t) * a.Hv + h;
        g_next = load_any(a.g, gi, a.g_dtype);
        b_next = load_any(a.beta, gi, a.beta_dtype);
      }
    };
    load_gates(0);
    uint32_t imma_phase = 0;
    for (int c = 0; c < nchunks; ++c) {
      const int slot = c & 1;
      float* sG = vec + (c % 3) * kVecSlot;
      float* sGam = sG + 64;
      float* sBeta = sG + 128;
      float* sDecay = sG + 192;
      const uint32_t kq = sb + kKQ + slot * kKQSlot;
      const uint32_t vt = sb + kV + slot * kVSlot;
      const uint32_t pt = sb + kP + slot * kPSlot;
      const uint32_t tmu = tmem + kTmU + slot * 64;
      float graw = g_next;
      if (it < kC) sBeta[it] = b_next;
      if (!group_wait(&bars[kBarKQV + slot], (c >> 1) & 1, kBarIntra, kIntraThreads)) break;
      TRACE(c, 0);
      if (it == 0) {
        tc::fence_after_sync();
#pragma unroll
        for (int s = 0; s < 8; ++s)
          tc::mma(tmem + kTmKQ, tc::kmajor_desc(kq, kKQBlock, s), tc::kmajor_desc(kq, kKQBlock, s),
                  kIdKQ, s > 0);
        tc::commit(&bars[kBarIMma]);
      }
      if (c + 1 < nchunks) load_gates(c + 1);
      // in-chunk cumulative log gate: threads 0..63 publish the raw gates, then
      // warp 0 scans them (lane l owns tokens 2l, 2l+1)
      if (it < kC) sG[it] = graw;
      tc::group_sync(kBarIntra, kIntraThreads);
      if (warp == 0) {
        const float g0 = sG[2 * lane], g1 = sG[2 * lane + 1];
        float run = g0 + g1;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const float o = __shfl_up_sync(0xffffffffu, run, off);
          if (lane >= off) run += o;
        }
        const float excl = run - (g0 + g1);
        const float GC = __shfl_sync(0xffffffffu, run, 31);
        __syncwarp();
        sG[2 * lane] = excl + g0;
        sG[2 * lane + 1] = run;
        sGam[2 * lane] = __expf(excl + g0);
        sGam[2 * lane + 1] = __expf(run);
        sDecay[2 * lane] = __expf(GC - (excl + g0));  // exp(G_C - G_j): V'' row scale
        sDecay[2 * lane + 1] = __expf(GC - run);
      }
      // P and U of this slot were last used by chunk c-2: wait until it is done
      if (c >= 2 && !group_wait(&bars[kBarSlotFree + slot], ((c - 2) >> 1) & 1, kBarIntra, kIntraThreads))
        break;
      if (!group_wait(&bars[kBarIMma], imma_phase, kBarIntra, kIntraThreads)) break;
      imma_phase ^= 1;
      tc::fence_after_sync();
      TRACE(c, 1);
      {  // A rows (TMEM lanes 0-63) and P rows (lanes 64-127); warps w and w+4
         // take columns [0, 32) and [32, 64)
        const int i = (quarter & 1) * 32 + lane;
        float r[32];
#pragma unroll
        for (int cb = 0; cb < 2; ++cb)
          tc::tmem_ld16(tmem + lane_base + kTmKQ + ih * 32 + cb * 16,
                        *reinterpret_cast<float(*)[16]>(r + cb * 16));
        tc::tmem_wait_ld();
        TRACE(c, 12);
        const float Gi = sG[i];
        if (quarter < 2) {
          const float bi = sBeta[i];
#pragma unroll
          for (int j4 = 0; j4 < 32; j4 += 4) {
            float4 v;
            float* pv = reinterpret_cast<float*>(&v);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int j = ih * 32 + j4 + e;
              pv[e] = (j < i) ? bi * __expf(Gi - sG[j]) * r[j4 + e] : 0.f;
            }
            *reinterpret_cast<float4*>(AT + i * kLd + ih * 32 + j4) = v;
          }
        } else {
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            const int j = ih * 32 + jj;
            r[jj] = (j <= i) ? r[jj] * __expf(Gi - sG[j]) : 0.f;
          }
          store_row16<BF16>(pt, i, ih * 4, r);
          store_row16<BF16>(pt, i, ih * 4 + 2, r + 16);
        }
      }
      TRACE(c, 13);
      tc::fence_before_sync();
      tc::group_sync(kBarIntra, kIntraThreads);
      TRACE(c, 2);
      solve_unit_lower(AT, Ms, warp, lane);
      TRACE(c, 3);
      {  // T_w = T diag(beta gamma), T_u = T diag(beta); thread: row i, 16 columns
        const int i = it >> 2, jq = it & 3;
        float tw[16], tu[16];
#pragma unroll
        for (int j4 = 0; j4 < 16; j4 += 4) {
          const float4 t4 = *reinterpret_cast<const float4*>(AT + i * kLd + jq * 16 + j4);
          const float tv[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = jq * 16 + j4 + e;
            const float t = (j <= i) ? tv[e] : 0.f;
            tu[j4 + e] = t * sBeta[j];
            tw[j4 + e] = tu[j4 + e] * sGam[j];
          }
        }
        store_row16<BF16>(sb + kTw, i, jq * 2, tw);
        store_row16<BF16>(sb + kTu, i, jq * 2, tu);
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      tc::group_sync(kBarIntra, kIntraThreads);
      TRACE(c, 4);
      if (it == 0) {  // W^T = K^T T_w^T (reuses the KQ columns), U^T = V^T T_u^T
        tc::fence_after_sync();
#pragma unroll
        for (int s = 0; s < 4; ++s)
          tc::mma(tmem + kTmKQ, tc::mnmajor_desc(kq, kKQBlock, s), tc::kmajor_desc(sb + kTw, 0, s),
                  kIdW, s > 0);
#pragma unroll
        for (int s = 0; s < 4; ++s)
          tc::mma(tmu, tc::mnmajor_desc(vt, kVBlock, s), tc::kmajor_desc(sb + kTu, 0, s), kIdW, s > 0);
        tc::commit(&bars[kBarIMma]);
      }
      // the W^T tile was read by the previous chunk's V' MMA: wait for it
      if (c >= 1 && !group_wait(&bars[kBarX], (c - 1) & 1, kBarIntra, kIntraThreads)) break;
      if (!group_wait(&bars[kBarIMma], imma_phase, kBarIntra, kIntraThreads)) break;
      imma_phase ^= 1;
      tc::fence_after_sync();
      TRACE(c, 5);
      {  // W^T -> bf16 tile, MN-major rows d_k = quarter*32 + lane, tokens [32 ih, +32)
        const int k = quarter * 32 + lane;
        float r[32];
#pragma unroll
        for (int cb = 0; cb < 2; ++cb)
          tc::tmem_ld16(tmem + lane_base + kTmKQ + ih * 32 + cb * 16,
                        *reinterpret_cast<float(*)[16]>(r + cb * 16));
        tc::tmem_wait_ld();
        store_row16<BF16>(sb + kWT, k, ih * 4, r);
        store_row16<BF16>(sb + kWT, k, ih * 4 + 2, r + 16);
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      mbar_arrive(&bars[kBarReady + slot]);
      TRACE(c, 6);
    }
  } else {
    // ================================================================ state
    asm volatile("setmaxnreg.inc.sync.aligned.u32 168;" ::: "memory");
    const int st = tid - kIntraThreads;  // 0..255
    const int quarter = warp & 3, half = (warp - kIntraThreads / 32) >> 2;
    const int dv = quarter * 32 + lane;
    const int k0 = half * 64;
    const size_t state_off = static_cast<size_t>(bh) * kD * kD;
    IO* o = static_cast<IO*>(a.o);
    float S[64];
#pragma unroll
    for (int j = 0; j < 64; ++j)
      S[j] = a.initial_state ? a.initial_state[state_off + static_cast<size_t>(k0 + j) * kD + dv] : 0.f;
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
    // outputs o[t0 + i][dv] = scale (gamma_i Z[dv][i] + O_intra[dv][i]): staged
    // as a [64][128] tile in the V''hi buffer (free between the previous
    // chunk's last MMA and this chunk's V'' epilogue), then written with
    // coalesced 16-byte stores
    auto outputs = [&](int c) {
      const float* sGam = vec + (c % 3) * kVecSlot + 64;
      IO* stage = reinterpret_cast<IO*>(smem + kVH);
      float z[32], oi[32];
      tc::tmem_ld16(tmem + lane_base + kTmZ + half * 32, *reinterpret_cast<float(*)[16]>(z));
      tc::tmem_ld16(tmem + lane_base + kTmZ + half * 32 + 16, *reinterpret_cast<float(*)[16]>(z + 16));
      tc::tmem_ld16(tmem + lane_base + kTmOI + half * 32, *reinterpret_cast<float(*)[16]>(oi));
      tc::tmem_ld16(tmem + lane_base + kTmOI + half * 32 + 16, *reinterpret_cast<float(*)[16]>(oi + 16));
      tc::tmem_wait_ld();
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const int i = half * 32 + jj;
        stage[i * kD + dv] = from_f32<IO>(a.scale * fmaf(sGam[i], z[jj], oi[jj]));
      }
      tc::fence_before_sync();
      tc::group_sync(kBarState, kStateThreads);
      const int t0 = c * kC;
#pragma unroll
      for (int r = 0; r < 4; ++r) {  // 64 rows x 256 B = 1024 16-byte pieces
        const int piece = r * kStateThreads + st;
        const int i = piece >> 4, col = (piece & 15) * 8;
        if (t0 + i < T) {
          const uint4 v = *reinterpret_cast<const uint4*>(stage + i * kD + col);
          *reinterpret_cast<uint4*>(o + ((static_cast<int64_t>(b) * T + t0 + i) * a.Hv + h) * kD + col) = v;
        }
      }
    };
    write_st();
    tc::group_sync(kBarState, kStateThreads);
    uint32_t x_phase = 0, z_phase = 0, s2_phase = 0;
    bool ok = true;
    for (int c = 0; c < nchunks; ++c) {
      const int slot = c & 1;
      const float* sG = vec + (c % 3) * kVecSlot;
      const float* sGam = sG + 64;
      const float* sDecay = sG + 192;
      const uint32_t kq = sb + kKQ + slot * kKQSlot;
      const uint32_t pt = sb + kP + slot * kPSlot;
      const uint32_t tmu = tmem + kTmU + slot * 64;
      if (!group_wait(&bars[kBarReady + slot], (c >> 1) & 1, kBarState, kStateThreads)) { ok = false; break; }
      TRACE(c, 7);
      if (st == 0) {  // V'^T = U^T - S^T W^T  (A = S^T from TMEM, negated)
        tc::fence_after_sync();
#pragma unroll
        for (int s = 0; s < 8; ++s)
          tc::mma_tmem_a(tmu, tmem + kTmST + s * 8, tc::mnmajor_desc(sb + kWT, 8192, s), kIdXneg, true);
        tc::commit(&bars[kBarX]);
      }
      if (c >= 1) {  // outputs of the previous chunk overlap the V' MMA
        if (!group_wait(&bars[kBarZ], z_phase, kBarState, kStateThreads)) { ok = false; break; }
        z_phase ^= 1;
        tc::fence_after_sync();
        outputs(c - 1);
      }
      tc::group_sync(kBarState, kStateThreads);
      if (st == 0) {  // Z^T = S^T Q^T
        tc::fence_after_sync();
#pragma unroll
        for (int s = 0; s < 8; ++s)
          tc::mma_tmem_a(tmem + kTmZ, tmem + kTmST + s * 8, tc::kmajor_desc(kq + 8192, kKQBlock, s),
                         kIdKQ, s > 0);
        tc::commit(&bars[kBarZ]);
      }
      if (!group_wait(&bars[kBarX], x_phase, kBarState, kStateThreads)) { ok = false; break; }
      x_phase ^= 1;
      tc::fence_after_sync();
      TRACE(c, 8);
      {  // V' (TMEM) -> bf16 V'^T tile; V'' = V' exp(G_C - G_j) -> hi / lo tiles
        float u[32];
        tc::tmem_ld16(tmu + lane_base + half * 32, *reinterpret_cast<float(*)[16]>(u));
        tc::tmem_ld16(tmu + lane_base + half * 32 + 16, *reinterpret_cast<float(*)[16]>(u + 16));
        tc::tmem_wait_ld();
#pragma unroll
        for (int cb = 0; cb < 2; ++cb) {
          // each pair is converted once; the packed hi word is reused for the
          // tile and unpacked for the lo residual
          uint32_t wp[8], wh[8], wl[8];
          const float4* dec4 = reinterpret_cast<const float4*>(sDecay + half * 32 + cb * 16);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const float4 d = dec4[q4];
            const float dd[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
            for (int e2 = 0; e2 < 2; ++e2) {
              const int e = q4 * 2 + e2;
              const float u0 = u[cb * 16 + 2 * e], u1 = u[cb * 16 + 2 * e + 1];
              const float v0 = u0 * dd[2 * e2], v1 = u1 * dd[2 * e2 + 1];
              wp[e] = tc::pack2<BF16>(u0, u1);
              wh[e] = tc::pack2<BF16>(v0, v1);
              wl[e] = tc::pack2<BF16>(v0 - tc::unpack_lo<BF16>(wh[e]), v1 - tc::unpack_hi<BF16>(wh[e]));
            }
          }
          const int ch = half * 4 + cb * 2;
#pragma unroll
          for (int k2 = 0; k2 < 2; ++k2) {
            tc::sts128(sb + kVP + tc::sw128_offset(dv, ch + k2), wp[4 * k2], wp[4 * k2 + 1],
                       wp[4 * k2 + 2], wp[4 * k2 + 3]);
            tc::sts128(sb + kVH + tc::sw128_offset(dv, ch + k2), wh[4 * k2], wh[4 * k2 + 1],
                       wh[4 * k2 + 2], wh[4 * k2 + 3]);
            tc::sts128(sb + kVL + tc::sw128_offset(dv, ch + k2), wl[4 * k2], wl[4 * k2 + 1],
                       wl[4 * k2 + 2], wl[4 * k2 + 3]);
          }
        }
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      tc::group_sync(kBarState, kStateThreads);
      TRACE(c, 9);
      if (st == 0) {  // O_intra^T = V'^T P^T ; dS^T = V''hi^T K + V''lo^T K
        tc::fence_after_sync();
#pragma unroll
        for (int s = 0; s < 4; ++s)
          tc::mma(tmem + kTmOI, tc::kmajor_desc(sb + kVP, 0, s), tc::kmajor_desc(pt, 0, s), kIdKQ, s > 0);
#pragma unroll
        for (int s = 0; s < 4; ++s)
          tc::mma(tmem + kTmDS, tc::kmajor_desc(sb + kVH, 0, s), tc::mnmajor_desc(kq, kKQBlock, s), kIdDS,
                  s > 0);
#pragma unroll
        for (int s = 0; s < 4; ++s)
          tc::mma(tmem + kTmDS, tc::kmajor_desc(sb + kVL, 0, s), tc::mnmajor_desc(kq, kKQBlock, s), kIdDS,
                  true);
        tc::commit(&bars[kBarS2]);
        tc::commit(&bars[kBarSlotFree + slot]);
      }
      if (!group_wait(&bars[kBarS2], s2_phase, kBarState, kStateThreads)) { ok = false; break; }
      s2_phase ^= 1;
      tc::fence_after_sync();
      if (st == 0 && c + 2 < nchunks) issue_tma(c + 2);  // this slot's MMAs are done
      TRACE(c, 10);
      {  // S <- gamma_C S + dS ; bf16 S^T back into TMEM for the next chunk
        const float gC = sGam[kC - 1];
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          float r[32];
          tc::tmem_ld16(tmem + lane_base + kTmDS + half * 64 + hb * 32, *reinterpret_cast<float(*)[16]>(r));
          tc::tmem_ld16(tmem + lane_base + kTmDS + half * 64 + hb * 32 + 16,
                        *reinterpret_cast<float(*)[16]>(r + 16));
          tc::tmem_wait_ld();
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) S[hb * 32 + jj] = fmaf(gC, S[hb * 32 + jj], r[jj]);
        }
        write_st();
      }
      tc::group_sync(kBarState, kStateThreads);
      TRACE(c, 11);
    }
    if (ok && nchunks > 0) {
      if (group_wait(&bars[kBarZ], z_phase, kBarState, kStateThreads)) {
        tc::fence_after_sync();
        outputs(nchunks - 1);
#pragma unroll
        for (int j = 0; j < 64; ++j)
          a.final_state[state_off + static_cast<size_t>(k0 + j) * kD + dv] = S[j];
      } else {
        ok = false;
      }
    }
    if (!ok && st == 0) {
      report(a.status, GDN_DEVERR_MMA_TIMEOUT);
      *abort_flag = 1;
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, kTmCols);
}

template <bool BF16>
int launch(const gdn_prefill_args_t& a, cudaStream_t stream) {
  static std::atomic<uint64_t> attr_done{0};
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  if (static_cast<int>(kSmemAlloc) > di.smem_optin) return GDN_ERR_SHAPE;
  auto kern = prefill_kernel<BF16>;
  rc = ensure_smem_attr(kern, kSmemAlloc, attr_done);
  if (rc) return rc;
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
  kern<<<static_cast<unsigned>(a.B * a.Hv), kThreads, kSmemAlloc, stream>>>(p, mq, mk, mv);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

int validate(const gdn_prefill_args_t* a) {
  if (!a) return GDN_ERR_NULL;
  if (!a->q || !a->k || !a->v || !a->g || !a->beta || !a->final_state || !a->o) return GDN_ERR_NULL;
  if (a->B < 1 || a->T < 1 || a->Hqk < 1 || a->Hv < 1 || a->Hv % a->Hqk) return GDN_ERR_SHAPE;
  if (a->dk != kD || a->dv != kD || a->chunk != kC) return GDN_ERR_SHAPE;
  if (static_cast<int64_t>(a->B) * a->Hv > 0x7FFFFFFF) return GDN_ERR_SHAPE;
  if (a->io_dtype != GDN_DT_BF16 && a->io_dtype != GDN_DT_F16) return GDN_ERR_DTYPE;
  if (!dtype_valid(a->g_dtype) || !dtype_valid(a->beta_dtype)) return GDN_ERR_DTYPE;
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->o) ||
      !aligned16(a->final_state) || (a->initial_state && !aligned16(a->initial_state)))
    return GDN_ERR_ALIGN;
  return GDN_OK;
}

}  // namespace prefill
}  // namespace gdn

#ifdef GDN_PREFILL_TRACE
extern "C" int gdn_prefill_trace_read(unsigned long long* host) {
  return cudaMemcpyFromSymbol(host, gdn::prefill::g_trace, sizeof(gdn::prefill::g_trace)) ==
                 cudaSuccess
             ? 0
             : 1;
}
#endif

extern "C" size_t gdn_prefill_workspace_size(const gdn_prefill_args_t*) { return 0; }

extern "C" int gdn_prefill_launch(const gdn_prefill_args_t* args, gdn_stream_t stream) {
  int rc = gdn::prefill::validate(args);
  if (rc) return rc;
  gdn::DeviceInfo di;
  if ((rc = gdn::device_info(&di))) return rc;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  return args->io_dtype == GDN_DT_BF16 ? gdn::prefill::launch<true>(*args, s)
                                       : gdn::prefill::launch<false>(*args, s);
}
