// gdn_decode.cu — GDN and KDA single-token decode for sm_100a.
//
// Math (per batch b, value head h; S is d_k x d_v fp32, row k, column v):
//     S_s = a * S            a = exp(g) scalar (GDN) or exp(g[k]) per row (KDA)
//     u   = k^T S_s          (one value per column)
//     r   = v - u
//     S'  = S_s + beta * k r^T
//     o   = scale * S'^T q = scale * (q^T S_s + beta * (q.k) * r)
// following gdn_decode_reference
// (analysis/wave15-attention-architecture/reference/pytorch_reference_gdn.py:38-91)
// and naive_recurrent_kda_step (pytorch_reference_kda.py:42-71).  The last
// identity lets one pass over S produce both column reductions, so the state
// crosses HBM exactly once in each direction.
//
// Work unit ("slab"): the DK x BV block of one head's state holding BV value
// columns.  Columns are independent, so slabs need no communication.
//
// Kernel structure (persistent, one CTA per SM, 9 warps):
//   warp 8 (producer): for each slab in the CTA's static schedule waits for a
//     free ring slot, then stages the slab plus the q/k rows, the v slice and
//     (KDA) the gate row into shared memory with cp.async.bulk, completing on
//     the slot's "full" mbarrier.  A contiguous slab (BV == d_v) is a single
//     1-D bulk copy; a column block (BV < d_v) is a single 2-D TMA tile copy
//     through a cached tensor map (one copy per row would serialise on the
//     copy engine: 128 small copies per slab).
//   warps 0-7 (consumers): wait "full", pull their rows of the slab into
//     registers with 16-byte shared loads, release the slot ("empty"), then
//     reduce k.S, q.S and q.k across rows (warp shuffles, then a ping-pong
//     shared buffer across warps), and write the updated rows straight back to
//     the state with 16-byte global stores (in place when state_out ==
//     state_in: each slab is read completely before any of it is written and
//     slabs are disjoint).
// Every mbarrier wait is bounded; a timeout sets a status bit and unwinds.
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>

#include "common.cuh"
#include "ptx.cuh"

namespace gdn {

struct DecodeParams {
  gdn_decode_args_t a;
  int64_t total_slabs;
  int32_t nvb;        // value-column blocks per head (d_v / BV)
  int32_t group;      // Hv / Hqk
  int32_t stages;     // ring depth
  int32_t stage_bytes;
  int32_t contiguous; // BV == d_v: a slab is one contiguous block
  int32_t g_row_bytes;
  int32_t has_peer;   // fused output all-gather (a.peer_out) in use
  gdn_peer_out_t po;  // its pointers, by value
};

// Acquire load of a flag another GPU writes (system scope).
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait (kWaitLimitNs) until every rank has released the output slot
// this step overwrites: free[j] >= step - 2 for all ranks j.
__device__ __forceinline__ bool peer_slots_free(const gdn_peer_out_t& po) {
  if (po.step < 3) return true;
  const uint32_t need = po.step - 2;
  const uint32_t* fr = po.free_flags[po.rank];
  const uint64_t t0 = global_timer_ns();
  for (int j = 0; j < po.n_ranks; ++j) {
    while (ld_acquire_sys(fr + j) < need) {
      if (global_timer_ns() - t0 > kWaitLimitNs) return false;
    }
  }
  return true;
}

// SB: bytes per state element (4 = fp32, the default; 2 = the optional fp16
// state, which halves the bytes a step streams).
template <int DK, int BV, bool KDA, int SB = 4>
struct DecodeTraits {
  // Small-batch variant (32-column slabs, d_k <= 128): 4 consumer warps and 4
  // CTAs per SM, so a small step's few slabs per SM run side by side instead of
  // one after another.
  static constexpr bool kSmall = BV == 32 && DK <= 128;
  static constexpr int kConsumerWarps = kSmall ? 4 : 8;
  static constexpr int kConsumers = kConsumerWarps * 32;
  static constexpr int kThreads = kConsumers + 32;
  static constexpr int kColGroups = BV / 4;                  // float4 columns
  static constexpr int kRowGroups = kConsumers / kColGroups;  // thread rows
  static constexpr int kRows = DK / kRowGroups;               // rows per thread
  static constexpr int kMaxStages = 8;
  // Narrow (32-column) slabs come with small batches, where a CTA walks a few
  // slabs back to back and each slab's reduction latency is exposed: those
  // variants run several CTAs per SM (fewer registers, a share of the smem).
  static constexpr int kCtasPerSm = kSmall ? 4 : (BV == 32 ? 2 : 1);
  static constexpr uint32_t kSlabBytes = DK * BV * SB;
  static constexpr uint32_t kQKBytes = DK * 2;
  static constexpr uint32_t kVBytes = BV * 2;
  static constexpr uint32_t kGBytes = KDA ? DK * 4 : 0;  // room for an fp32 gate row
  static constexpr uint32_t kStageBytes =
      (kSlabBytes + 2 * kQKBytes + kVBytes + kGBytes + 127) / 128 * 128;
  // header: 2*8 mbarriers + abort flag (256 B), then the reduction buffers
  static constexpr uint32_t kRedFloats = 2 * kConsumerWarps * BV * 2 + 2 * kConsumerWarps;
  static constexpr uint32_t kHeaderBytes = (256 + kRedFloats * 4 + 127) / 128 * 128;
  static_assert(kColGroups <= 32 && 32 % kColGroups == 0, "BV must be 32..128");
  static_assert(DK % kRowGroups == 0, "DK must be a multiple of the row groups");
};

// PRE: the fused layer-preprocessing variant (in-kernel q/k L2 norm, gate from
// the raw projection), a separate instantiation so the plain kernel carries
// none of its code.
template <int DK, int BV, typename IO, bool KDA, bool PRE, int SB>
__global__ void __launch_bounds__(DecodeTraits<DK, BV, KDA, SB>::kThreads,
                                  DecodeTraits<DK, BV, KDA, SB>::kCtasPerSm)
    decode_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap state_map) {
  using Tr = DecodeTraits<DK, BV, KDA, SB>;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + Tr::kMaxStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + Tr::kMaxStages);
  float* red = reinterpret_cast<float*>(smem + 256);  // [2][warps][2][BV]
  float* red_qk = red + 2 * Tr::kConsumerWarps * BV * 2;  // [2][warps]
  unsigned char* ring = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem + Tr::kHeaderBytes) + 127) & ~uintptr_t(127));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const gdn_decode_args_t& a = p.a;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], Tr::kConsumerWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // The prologue above may overlap the previous kernel in the stream; every
  // global access below comes after it has completed (inputs and the state
  // may be its outputs).
  pdl_launch_dependents();
  pdl_wait();

  if (warp == Tr::kConsumerWarps) {
    // ------------------------------------------------------------ producer
    int it = 0;
    for (int64_t slab = blockIdx.x; slab < p.total_slabs; slab += gridDim.x, ++it) {
      const int stage = it % p.stages;
      const uint32_t round = it / p.stages;
      int ok = 1;
      if (lane == 0) ok = mbar_wait_bounded(&empty[stage], (round & 1) ^ 1);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok || *abort_flag) {
        if (!ok && lane == 0) {
          report(a.status, GDN_DEVERR_EMPTY_TIMEOUT);
          *abort_flag = 1;
        }
        break;
      }
      const int64_t bh = slab / p.nvb;
      const int vb = static_cast<int>(slab - bh * p.nvb);
      const int64_t b = bh / a.Hv;
      const int h = static_cast<int>(bh - b * a.Hv);
      const int hq = h / p.group;
      unsigned char* st = ring + static_cast<size_t>(stage) * p.stage_bytes;
      const unsigned char* src = reinterpret_cast<const unsigned char*>(a.state_in) +
                                 ((bh * DK) * a.dv + static_cast<int64_t>(vb) * BV) * SB;
      if (lane == 0) {
        uint32_t bytes = 2 * Tr::kQKBytes + Tr::kVBytes + Tr::kSlabBytes;
        if (KDA) bytes += p.g_row_bytes;
        mbar_expect_tx(&full[stage], bytes);
        const IO* q = static_cast<const IO*>(a.q) + b * a.q_sb + static_cast<int64_t>(hq) * a.q_sh;
        const IO* k = static_cast<const IO*>(a.k) + b * a.k_sb + static_cast<int64_t>(hq) * a.k_sh;
        const IO* v = static_cast<const IO*>(a.v) + b * a.v_sb + static_cast<int64_t>(h) * a.v_sh +
                      static_cast<int64_t>(vb) * BV;
        bulk_g2s(st + Tr::kSlabBytes, q, Tr::kQKBytes, &full[stage]);
        bulk_g2s(st + Tr::kSlabBytes + Tr::kQKBytes, k, Tr::kQKBytes, &full[stage]);
        bulk_g2s(st + Tr::kSlabBytes + 2 * Tr::kQKBytes, v, Tr::kVBytes, &full[stage]);
        if (KDA) {
          const unsigned char* g = static_cast<const unsigned char*>(a.g) +
                                   (b * a.g_sb + static_cast<int64_t>(h) * a.g_sh) *
                                       (a.g_dtype == GDN_DT_F32 ? 4 : 2);
          bulk_g2s(st + Tr::kSlabBytes + 2 * Tr::kQKBytes + Tr::kVBytes, g, p.g_row_bytes,
                   &full[stage]);
        }
        if (p.contiguous)
          bulk_g2s(st, src, Tr::kSlabBytes, &full[stage]);
        else  // x = first column (vb*BV*4 bytes: 16-byte aligned), y = first row
          tma_load_2d(st, &state_map, vb * BV, static_cast<int>(bh * DK), &full[stage]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[stage]);
    }
    // On abort, copies issued into slots the consumers never drained may still
    // be in flight: wait (bounded) for them before the CTA's shared memory is
    // released.
    if (*abort_flag && lane == 0) {
      const int n = it < p.stages ? it : p.stages;
      for (int j = 0; j < n; ++j) {
        const int jt = it - 1 - j;
        if (jt < 0) break;
        if (!mbar_wait_bounded(&full[jt % p.stages], (jt / p.stages) & 1)) {
          report(a.status, GDN_DEVERR_DRAIN_TIMEOUT);
          break;
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int tid = threadIdx.x;                 // 0 .. kConsumers-1
  const int cg = tid % Tr::kColGroups;         // float4 column group
  const int rg = tid / Tr::kColGroups;         // first row of this thread
  const float scale = a.scale;
  // fused all-gather: this rank has consumed step - 1 (its reads of gathered
  // outputs precede this launch), so tell every rank
  if (p.has_peer && blockIdx.x == 0 && tid == 0) {
    for (int j = 0; j < p.po.n_ranks; ++j)
      atomicMax_system(p.po.free_flags[j] + p.po.rank, p.po.step - 1);
  }
  bool peer_ok = p.has_peer != 0;  // peer stores allowed (slot released)
  bool peer_checked = false;
  int it = 0;
  for (int64_t slab = blockIdx.x; slab < p.total_slabs; slab += gridDim.x, ++it) {
    const int stage = it % p.stages;
    const uint32_t round = it / p.stages;
    const int64_t bh = slab / p.nvb;
    const int vb = static_cast<int>(slab - bh * p.nvb);
    const int64_t b = bh / a.Hv;
    const int h = static_cast<int>(bh - b * a.Hv);

    // per-(b,h) scalars: issued before the wait so their latency overlaps it
    const float beta = load_any(a.beta, b * a.beta_sb + static_cast<int64_t>(h) * a.beta_sh,
                                a.beta_dtype);
    float alpha = 1.f;
    if (!KDA) {
      const float g = load_any(a.g, b * a.g_sb + static_cast<int64_t>(h) * a.g_sh, a.g_dtype);
      if (PRE && (a.flags & GDN_DECODE_GATE_RAW)) {
        // log gate from the raw projection: -exp(A_log) * softplus(a + dt_bias)
        const float x = g + __ldg(a.dt_bias + h);
        const float sp = x > 20.f ? x : log1pf(expf(x));
        alpha = expf(-expf(__ldg(a.A_log + h)) * sp);
      } else {
        alpha = (a.gate_kind == GDN_GATE_LOG) ? __expf(g) : g;
      }
    }

    // output norm/gate operand z (fused layer step), fetched while the slab lands
    float zf[4] = {0.f, 0.f, 0.f, 0.f};
    if (PRE && (a.flags & GDN_DECODE_OUT_NORM_GATE) && rg == 0) {
      const IO* zp = static_cast<const IO*>(a.z) + b * a.z_sb + static_cast<int64_t>(h) * a.z_sh +
                     static_cast<int64_t>(vb) * BV + cg * 4;
      const uint2 w = __ldg(reinterpret_cast<const uint2*>(zp));
      const IO* zv = reinterpret_cast<const IO*>(&w);
#pragma unroll
      for (int e = 0; e < 4; ++e) zf[e] = to_f32(zv[e]);
    }

    // A timed-out thread still runs to the reduction barrier below, where the
    // consumers agree (bar.red.or) to stop together; no thread is left behind
    // on a barrier.
    const bool landed = mbar_wait_bounded(&full[stage], round & 1);
    const unsigned char* st = ring + static_cast<size_t>(stage) * p.stage_bytes;
    const float* s_slab = reinterpret_cast<const float*>(st);
    const IO* s_q = reinterpret_cast<const IO*>(st + Tr::kSlabBytes);
    const IO* s_k = reinterpret_cast<const IO*>(st + Tr::kSlabBytes + Tr::kQKBytes);
    const IO* s_v = reinterpret_cast<const IO*>(st + Tr::kSlabBytes + 2 * Tr::kQKBytes);
    const void* s_g = st + Tr::kSlabBytes + 2 * Tr::kQKBytes + Tr::kVBytes;

    float4 s[Tr::kRows];
    float kr[Tr::kRows];
    float4 u = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 qs = make_float4(0.f, 0.f, 0.f, 0.f);
    float qk = 0.f;
#pragma unroll
    for (int i = 0; i < Tr::kRows; ++i) {
      const int row = rg + i * Tr::kRowGroups;
      float4 x;
      if (SB == 4) {
        x = lds128(s_slab + row * BV + cg * 4);
      } else {  // fp16 state: 4 halves (8 bytes), widened to fp32
        const uint2 w = *reinterpret_cast<const uint2*>(st + (row * BV + cg * 4) * 2);
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
        x = make_float4(lo.x, lo.y, hi.x, hi.y);
      }
      const float kv = to_f32(s_k[row]);
      const float qv = to_f32(s_q[row]);
      float ai = alpha;
      if (KDA) {
        const float gr = smem_any(s_g, row, a.g_dtype);
        ai = (a.gate_kind == GDN_GATE_LOG) ? __expf(gr) : gr;
      }
      x.x *= ai; x.y *= ai; x.z *= ai; x.w *= ai;
      u.x = fmaf(kv, x.x, u.x); u.y = fmaf(kv, x.y, u.y);
      u.z = fmaf(kv, x.z, u.z); u.w = fmaf(kv, x.w, u.w);
      qs.x = fmaf(qv, x.x, qs.x); qs.y = fmaf(qv, x.y, qs.y);
      qs.z = fmaf(qv, x.z, qs.z); qs.w = fmaf(qv, x.w, qs.w);
      qk = fmaf(qv, kv, qk);
      s[i] = x;
      kr[i] = kv;
    }
    float4 vv;
    vv.x = to_f32(s_v[cg * 4 + 0]);
    vv.y = to_f32(s_v[cg * 4 + 1]);
    vv.z = to_f32(s_v[cg * 4 + 2]);
    vv.w = to_f32(s_v[cg * 4 + 3]);
    // |q|^2 and |k|^2 for the in-kernel L2 normalisation: every warp sums the
    // staged rows itself (no extra state in the row loop, nothing when off)
    float qq = 0.f, kk = 0.f;
    if (PRE && (a.flags & GDN_DECODE_L2NORM_QK)) {
#pragma unroll
      for (int e = lane; e < DK; e += 32) {
        const float qe = to_f32(s_q[e]), ke = to_f32(s_k[e]);
        qq = fmaf(qe, qe, qq);
        kk = fmaf(ke, ke, kk);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        qq += __shfl_xor_sync(0xffffffffu, qq, off);
        kk += __shfl_xor_sync(0xffffffffu, kk, off);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);  // slot may be refilled now

    // reduce over the row groups inside this warp
#pragma unroll
    for (int off = Tr::kColGroups; off < 32; off <<= 1) {
      u.x += __shfl_xor_sync(0xffffffffu, u.x, off);
      u.y += __shfl_xor_sync(0xffffffffu, u.y, off);
      u.z += __shfl_xor_sync(0xffffffffu, u.z, off);
      u.w += __shfl_xor_sync(0xffffffffu, u.w, off);
      qs.x += __shfl_xor_sync(0xffffffffu, qs.x, off);
      qs.y += __shfl_xor_sync(0xffffffffu, qs.y, off);
      qs.z += __shfl_xor_sync(0xffffffffu, qs.z, off);
      qs.w += __shfl_xor_sync(0xffffffffu, qs.w, off);
      qk += __shfl_xor_sync(0xffffffffu, qk, off);
    }
    // ... then across warps through a ping-pong buffer (one barrier per slab)
    float* rb = red + (it & 1) * (Tr::kConsumerWarps * BV * 2);
    float* rq = red_qk + (it & 1) * Tr::kConsumerWarps;
    if (lane < Tr::kColGroups) {
      *reinterpret_cast<float4*>(rb + warp * BV * 2 + cg * 4) = u;
      *reinterpret_cast<float4*>(rb + warp * BV * 2 + BV + cg * 4) = qs;
    }
    if (lane == 0) rq[warp] = qk;
    if (named_barrier_or(1, Tr::kConsumers, !landed)) {
      if (!landed) report(a.status, GDN_DEVERR_FULL_TIMEOUT);
      *abort_flag = 1;
      break;
    }
    u = make_float4(0.f, 0.f, 0.f, 0.f);
    qs = make_float4(0.f, 0.f, 0.f, 0.f);
    qk = 0.f;
#pragma unroll
    for (int w = 0; w < Tr::kConsumerWarps; ++w) {
      const float4 pu = *reinterpret_cast<const float4*>(rb + w * BV * 2 + cg * 4);
      const float4 pq = *reinterpret_cast<const float4*>(rb + w * BV * 2 + BV + cg * 4);
      u.x += pu.x; u.y += pu.y; u.z += pu.z; u.w += pu.w;
      qs.x += pq.x; qs.y += pq.y; qs.z += pq.z; qs.w += pq.w;
      qk += rq[w];
    }
    // In-kernel L2 normalisation of q and k folds into the reduced scalars:
    // every use of k (u, q.k, the update beta k r^T) and of q (q.S, q.k) is
    // linear in it.
    float rk = 1.f, rqn = 1.f;
    if (PRE && (a.flags & GDN_DECODE_L2NORM_QK)) {
      rk = rsqrtf(kk + a.l2_eps);
      rqn = rsqrtf(qq + a.l2_eps);
      u.x *= rk; u.y *= rk; u.z *= rk; u.w *= rk;
      qs.x *= rqn; qs.y *= rqn; qs.z *= rqn; qs.w *= rqn;
      qk *= rqn * rk;
    }
    float4 r;
    r.x = vv.x - u.x; r.y = vv.y - u.y; r.z = vv.z - u.z; r.w = vv.w - u.w;

    if (rg == 0) {
      const float bqk = beta * qk;
      float of[4];
      of[0] = scale * fmaf(bqk, r.x, qs.x);
      of[1] = scale * fmaf(bqk, r.y, qs.y);
      of[2] = scale * fmaf(bqk, r.z, qs.z);
      of[3] = scale * fmaf(bqk, r.w, qs.w);
      if (PRE && (a.flags & GDN_DECODE_OUT_NORM_GATE)) {
        // the slab is the whole d_v row (BV == d_v): these kColGroups lanes of
        // warp 0 hold the head's complete output
        float ss = of[0] * of[0] + of[1] * of[1] + of[2] * of[2] + of[3] * of[3];
        constexpr unsigned kMask = Tr::kColGroups == 32 ? 0xffffffffu : ((1u << Tr::kColGroups) - 1u);
#pragma unroll
        for (int off = Tr::kColGroups / 2; off > 0; off >>= 1) ss += __shfl_xor_sync(kMask, ss, off);
        const float rstd = rsqrtf(ss / static_cast<float>(BV) + a.norm_eps);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float silu = zf[e] / (1.f + __expf(-zf[e]));
          of[e] = of[e] * rstd * __ldg(a.norm_weight + cg * 4 + e) * silu;
        }
      }
      IO ov[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) ov[e] = from_f32<IO>(of[e]);
      const int64_t off = b * a.o_sb + static_cast<int64_t>(h) * a.o_sh + static_cast<int64_t>(vb) * BV + cg * 4;
      IO* o = static_cast<IO*>(a.o) + off;
      *reinterpret_cast<uint2*>(o) = *reinterpret_cast<const uint2*>(ov);
      if (peer_ok) {
        // the output-writing lanes (0 .. kColGroups-1 of warp 0) agree on one
        // bounded wait for the slot, done once per CTA by lane 0
        constexpr unsigned kMask = Tr::kColGroups == 32 ? 0xffffffffu : ((1u << Tr::kColGroups) - 1u);
        if (!peer_checked) {
          peer_checked = true;
          int okw = 1;
          if (cg == 0) {
            okw = peer_slots_free(p.po) ? 1 : 0;
            if (!okw) report(a.status, GDN_DEVERR_PEER_TIMEOUT);
          }
          peer_ok = __shfl_sync(kMask, okw, 0) != 0;
        }
        if (peer_ok) {  // 16-byte stores: even lanes send their and their neighbour's 4 outputs
          const uint2 mine = *reinterpret_cast<const uint2*>(ov);
          const uint32_t nx = __shfl_xor_sync(kMask, mine.x, 1);
          const uint32_t ny = __shfl_xor_sync(kMask, mine.y, 1);
          if ((cg & 1) == 0) {
            const uint4 w = make_uint4(mine.x, mine.y, nx, ny);
            for (int i = 0; i < p.po.n_ranks - 1; ++i)
              *reinterpret_cast<uint4*>(static_cast<IO*>(p.po.o_peer[i]) + off) = w;
          }
        }
      }
    }

    unsigned char* dst = reinterpret_cast<unsigned char*>(a.state_out) +
                         ((bh * DK) * a.dv + static_cast<int64_t>(vb) * BV + cg * 4) * SB;
#pragma unroll
    for (int i = 0; i < Tr::kRows; ++i) {
      const int row = rg + i * Tr::kRowGroups;
      const float bk = PRE ? beta * rk * kr[i] : beta * kr[i];
      float4 x = s[i];
      x.x = fmaf(bk, r.x, x.x); x.y = fmaf(bk, r.y, x.y);
      x.z = fmaf(bk, r.z, x.z); x.w = fmaf(bk, r.w, x.w);
      unsigned char* drow = dst + static_cast<int64_t>(row) * a.dv * SB;
      if (SB == 4) {
        stg128(reinterpret_cast<float*>(drow), x);
      } else {
        const __half2 lo = __floats2half2_rn(x.x, x.y), hi = __floats2half2_rn(x.z, x.w);
        asm volatile("st.global.v2.b32 [%0], {%1, %2};" ::"l"(drow),
                     "r"(*reinterpret_cast<const uint32_t*>(&lo)),
                     "r"(*reinterpret_cast<const uint32_t*>(&hi))
                     : "memory");
      }
    }
  }
  if (p.has_peer) {
    // every output store of this CTA (local and remote) is made visible at
    // system scope before the CTA counts itself done; the last CTA of the
    // grid then adds 1 to every rank's arrival counter
    __threadfence_system();
    const bool aborted = named_barrier_or(1, Tr::kConsumers, *abort_flag != 0);
    if (tid == 0 && !aborted) {
      const uint32_t old = atomicAdd(p.po.cta_done, 1u);
      if (old + 1u == p.po.step * gridDim.x) {
        __threadfence_system();
        for (int j = 0; j < p.po.n_ranks; ++j) atomicAdd_system(p.po.arrive[j], 1u);
      }
    }
  }
}

// ------------------------------------------------------------------ launcher

template <int DK, int BV, typename IO, bool KDA, bool PRE, int SB>
static int launch_decode_impl(const gdn_decode_args_t& a, cudaStream_t stream) {
  using Tr = DecodeTraits<DK, BV, KDA, SB>;
  static std::atomic<uint64_t> attr_done{0};
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc) return rc;
  const int smem_budget = Tr::kCtasPerSm == 1 ? di.smem_optin
                                              : di.smem_per_sm / Tr::kCtasPerSm - 1024;
  int stages =
      (smem_budget - static_cast<int>(Tr::kHeaderBytes) - 128) / static_cast<int>(Tr::kStageBytes);
  if (stages > Tr::kMaxStages) stages = Tr::kMaxStages;
  if (stages < 2) return GDN_ERR_SHAPE;
  const int smem = Tr::kHeaderBytes + 128 + stages * Tr::kStageBytes;
  auto kern = decode_kernel<DK, BV, IO, KDA, PRE, SB>;
  rc = ensure_smem_attr(kern, smem, attr_done);
  if (rc) return rc;

  DecodeParams p;
  p.a = a;
  p.nvb = a.dv / BV;
  p.total_slabs = static_cast<int64_t>(a.B) * a.Hv * p.nvb;
  p.group = a.Hv / a.Hqk;
  p.stages = stages;
  p.stage_bytes = Tr::kStageBytes;
  p.contiguous = (BV == a.dv) ? 1 : 0;
  p.g_row_bytes = KDA ? DK * host_dtype_size(a.g_dtype) : 0;
  p.has_peer = a.peer_out ? 1 : 0;
  if (a.peer_out) p.po = *a.peer_out;
  else std::memset(&p.po, 0, sizeof(p.po));
  CUtensorMap map;
  std::memset(&map, 0, sizeof(map));
  if (!p.contiguous) {
    const uint64_t dims[2] = {static_cast<uint64_t>(a.dv), static_cast<uint64_t>(a.B) * a.Hv * DK};
    const uint64_t strides[1] = {static_cast<uint64_t>(a.dv) * SB};
    const uint32_t box[2] = {BV, DK};
    rc = tensor_map(&map, SB == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                    2, a.state_in, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  int ctas = (di.sm_count - (a.sm_reserve > 0 ? a.sm_reserve : 0)) * Tr::kCtasPerSm;
  if (ctas < 1) ctas = 1;
  const int64_t grid64 = p.total_slabs < ctas ? p.total_slabs : ctas;
  // programmatic dependent launch: this kernel's prologue (barrier set-up)
  // overlaps the tail of the previous kernel in the stream
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid64));
  cfg.blockDim = dim3(Tr::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, p, map) != cudaSuccess) {
    (void)cudaGetLastError();
    return GDN_ERR_LAUNCH;
  }
  return GDN_OK;
}

static int validate_decode(const gdn_decode_args_t* a, bool kda) {
  if (!a) return GDN_ERR_NULL;
  if (!a->q || !a->k || !a->v || !a->g || !a->beta || !a->state_in || !a->state_out || !a->o)
    return GDN_ERR_NULL;
  if (a->B < 1 || a->Hqk < 1 || a->Hv < 1 || a->Hv % a->Hqk) return GDN_ERR_SHAPE;
  if (a->dk != 64 && a->dk != 128 && a->dk != 256) return GDN_ERR_SHAPE;
  if (a->dv < 64 || a->dv % 64) return GDN_ERR_SHAPE;
  if (a->io_dtype != GDN_DT_BF16 && a->io_dtype != GDN_DT_F16) return GDN_ERR_DTYPE;
  if (!dtype_valid(a->g_dtype) || !dtype_valid(a->beta_dtype)) return GDN_ERR_DTYPE;
  if (a->gate_kind != GDN_GATE_LOG && a->gate_kind != GDN_GATE_LINEAR) return GDN_ERR_DTYPE;
  if (a->flags & ~(GDN_DECODE_L2NORM_QK | GDN_DECODE_GATE_RAW | GDN_DECODE_OUT_NORM_GATE))
    return GDN_ERR_DTYPE;
  if (a->flags & GDN_DECODE_OUT_NORM_GATE) {
    if (!a->z || !a->norm_weight) return GDN_ERR_NULL;
    if ((a->dv != 64 && a->dv != 128) || a->dk > 128 || (a->dk == 64 && a->dv != 64))
      return GDN_ERR_SHAPE;
    if (!aligned16(a->z) || !stride_ok(a->z_sb, 2) || !stride_ok(a->z_sh, 2)) return GDN_ERR_ALIGN;
  }
  if (a->state_dtype != GDN_DT_F32 && a->state_dtype != GDN_DT_F16) return GDN_ERR_DTYPE;
  if (a->peer_out) {
    const gdn_peer_out_t& po = *a->peer_out;
    if (po.n_ranks < 2 || po.n_ranks > 8 || po.rank < 0 || po.rank >= po.n_ranks || po.step < 1)
      return GDN_ERR_SHAPE;
    if (!po.cta_done) return GDN_ERR_NULL;
    for (int j = 0; j < po.n_ranks; ++j)
      if (!po.arrive[j] || !po.free_flags[j]) return GDN_ERR_NULL;
    for (int i = 0; i < po.n_ranks - 1; ++i)
      if (!po.o_peer[i] || !aligned16(po.o_peer[i])) return GDN_ERR_NULL;
  }
  if (a->flags & GDN_DECODE_GATE_RAW) {
    if (kda) return GDN_ERR_DTYPE;  // the raw-gate formula is the scalar GDN gate
    if (!a->A_log || !a->dt_bias) return GDN_ERR_NULL;
  }
  if ((a->flags & GDN_DECODE_L2NORM_QK) && !(a->l2_eps >= 0.f)) return GDN_ERR_SHAPE;
  // bulk-copied rows: 16-byte aligned bases and strides
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->o) ||
      !aligned16(a->state_in) || !aligned16(a->state_out))
    return GDN_ERR_ALIGN;
  if (!stride_ok(a->q_sb, 2) || !stride_ok(a->q_sh, 2) || !stride_ok(a->k_sb, 2) ||
      !stride_ok(a->k_sh, 2) || !stride_ok(a->v_sb, 2) || !stride_ok(a->v_sh, 2) ||
      !stride_ok(a->o_sb, 2) || !stride_ok(a->o_sh, 2))
    return GDN_ERR_ALIGN;
  if (kda) {
    const int gs = host_dtype_size(a->g_dtype);
    if (!aligned16(a->g) || !stride_ok(a->g_sb, gs) || !stride_ok(a->g_sh, gs)) return GDN_ERR_ALIGN;
  }
  // in place, or fully disjoint
  if (a->state_in != a->state_out) {
    const size_t n = static_cast<size_t>(a->B) * a->Hv * a->dk * a->dv *
                     (a->state_dtype == GDN_DT_F16 ? 2 : 4);
    const char* i0 = reinterpret_cast<const char*>(a->state_in);
    const char* o0 = reinterpret_cast<const char*>(a->state_out);
    if (i0 < o0 + n && o0 < i0 + n) return GDN_ERR_SHAPE;
  }
  return GDN_OK;
}

// Chooses the value-column block: the widest block (whole rows when possible,
// a single contiguous copy) that still gives every SM at least four slabs;
// small batches fall back to narrower blocks for balance.
static int pick_bv(const gdn_decode_args_t& a, int sm_count) {
  if (a.flags & GDN_DECODE_OUT_NORM_GATE) return a.dv;  // the norm needs whole rows
  static const int kAllowed128[] = {128, 64, 32};
  static const int kAllowed256[] = {64, 32};
  const int* allowed = a.dk == 256 ? kAllowed256 : kAllowed128;
  const int n = a.dk == 256 ? 2 : 3;
  if (a.dk == 64) return 64;
  int last = 0;
  for (int i = 0; i < n; ++i) {
    const int bv = allowed[i];
    if (a.dv % bv) continue;
    last = bv;
    const int64_t slabs = static_cast<int64_t>(a.B) * a.Hv * (a.dv / bv);
    if (slabs >= 4 * static_cast<int64_t>(sm_count)) return bv;
  }
  return last;
}

template <typename IO, bool KDA, bool PRE>
static int dispatch_dk(const gdn_decode_args_t& a, cudaStream_t stream, int bv) {
  if (a.state_dtype == GDN_DT_F16) {  // fp16 state: d = 128 only
    if (a.dk != 128) return GDN_ERR_SHAPE;
    if (bv == 128) return launch_decode_impl<128, 128, IO, KDA, PRE, 2>(a, stream);
    if (bv == 64) return launch_decode_impl<128, 64, IO, KDA, PRE, 2>(a, stream);
    return launch_decode_impl<128, 32, IO, KDA, PRE, 2>(a, stream);
  }
  switch (a.dk) {
    case 64: return launch_decode_impl<64, 64, IO, KDA, PRE, 4>(a, stream);
    case 128:
      if (bv == 128) return launch_decode_impl<128, 128, IO, KDA, PRE, 4>(a, stream);
      if (bv == 64) return launch_decode_impl<128, 64, IO, KDA, PRE, 4>(a, stream);
      return launch_decode_impl<128, 32, IO, KDA, PRE, 4>(a, stream);
    case 256:
      return bv == 64 ? launch_decode_impl<256, 64, IO, KDA, PRE, 4>(a, stream)
                      : launch_decode_impl<256, 32, IO, KDA, PRE, 4>(a, stream);
  }
  return GDN_ERR_SHAPE;
}

template <typename IO, bool KDA>
static int dispatch_pre(const gdn_decode_args_t& a, cudaStream_t stream, int bv) {
  return a.flags ? dispatch_dk<IO, KDA, true>(a, stream, bv) : dispatch_dk<IO, KDA, false>(a, stream, bv);
}

static int decode_entry(const gdn_decode_args_t* a, cudaStream_t stream, bool kda) {
  int rc = validate_decode(a, kda);
  if (rc) return rc;
  DeviceInfo di;
  rc = device_info(&di);
  if (rc) return rc;
  const int bv = pick_bv(*a, di.sm_count);
  if (a->io_dtype == GDN_DT_BF16)
    return kda ? dispatch_pre<__nv_bfloat16, true>(*a, stream, bv)
               : dispatch_pre<__nv_bfloat16, false>(*a, stream, bv);
  return kda ? dispatch_pre<__half, true>(*a, stream, bv) : dispatch_pre<__half, false>(*a, stream, bv);
}

}  // namespace gdn

extern "C" int gdn_decode_launch(const gdn_decode_args_t* args, gdn_stream_t stream) {
  return gdn::decode_entry(args, reinterpret_cast<cudaStream_t>(stream), false);
}

extern "C" int kda_decode_launch(const gdn_decode_args_t* args, gdn_stream_t stream) {
  return gdn::decode_entry(args, reinterpret_cast<cudaStream_t>(stream), true);
}

static gdn_decode_args_t ref_layout_args(int32_t B, int32_t H, int32_t dk, int32_t dv,
                                         const void* dQ, const void* dK, const void* dV,
                                         const void* dG, const void* dBeta, const float* dS_in,
                                         float* dS_out, void* dO, int32_t io_dtype, bool kda) {
  gdn_decode_args_t a{};
  a.q = dQ; a.k = dK; a.v = dV; a.g = dG; a.beta = dBeta;
  a.state_in = dS_in; a.state_out = dS_out; a.o = dO;
  a.q_sb = static_cast<int64_t>(H) * dk; a.q_sh = dk;
  a.k_sb = a.q_sb; a.k_sh = dk;
  a.v_sb = static_cast<int64_t>(H) * dv; a.v_sh = dv;
  a.o_sb = a.v_sb; a.o_sh = dv;
  a.g_sb = kda ? static_cast<int64_t>(H) * dk : H; a.g_sh = kda ? dk : 1;
  a.beta_sb = H; a.beta_sh = 1;
  a.B = B; a.Hqk = H; a.Hv = H; a.dk = dk; a.dv = dv;
  a.io_dtype = io_dtype; a.g_dtype = io_dtype; a.beta_dtype = io_dtype;
  a.gate_kind = kda ? GDN_GATE_LOG : GDN_GATE_LINEAR;
  a.scale = 1.0f;
  a.status = nullptr;
  return a;
}

extern "C" int gdn_decode_ref_launch(int32_t B, int32_t H, int32_t dk, int32_t dv, const void* dQ,
                                     const void* dK, const void* dV, const void* dAlpha,
                                     const void* dBeta, const float* dS_in, float* dS_out, void* dO,
                                     int32_t io_dtype, gdn_stream_t stream) {
  const gdn_decode_args_t a =
      ref_layout_args(B, H, dk, dv, dQ, dK, dV, dAlpha, dBeta, dS_in, dS_out, dO, io_dtype, false);
  return gdn_decode_launch(&a, stream);
}

extern "C" int kda_decode_ref_launch(int32_t B, int32_t H, int32_t dk, int32_t dv, const void* dQ,
                                     const void* dK, const void* dV, const void* dG,
                                     const void* dBeta, const float* dS_in, float* dS_out, void* dO,
                                     int32_t io_dtype, gdn_stream_t stream) {
  const gdn_decode_args_t a =
      ref_layout_args(B, H, dk, dv, dQ, dK, dV, dG, dBeta, dS_in, dS_out, dO, io_dtype, true);
  return kda_decode_launch(&a, stream);
}
