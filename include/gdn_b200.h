/*
 * gdn_b200.h — C ABI of the B200 (sm_100a) gated delta-rule library.
 *
 * The library implements three operations of the gated delta rule
 * (GDN / KDA linear attention), each as hand-written sm_100a CUDA:
 *
 *   GDN decode (one token per sequence, scalar gate per head)
 *       S      <- a * S                      a = exp(g) (log gate) or g (linear gate)
 *       u      =  k^T S                       (per value column)
 *       S      <- S + beta * k (v - u)^T
 *       o      =  scale * S^T q
 *   KDA decode: identical, but the gate is a d_k-vector, S <- diag(exp(g)) S.
 *   GDN chunked prefill: the same recurrence over T tokens, computed chunk by
 *       chunk (WY / UT transform) on the tcgen05 tensor cores.
 *
 * Conventions shared by every entry point
 *   - Every pointer is a DEVICE pointer on the current CUDA device.  The caller
 *     owns all memory; no entry point allocates device memory.
 *   - The state is fp32, laid out [B, Hv, d_k, d_v] row-major (S[k][v]), and is
 *     updated in place when state_out == state_in.
 *   - q/k have Hqk heads, v/o/g/beta have Hv heads; Hv must be a multiple of
 *     Hqk and value head h reads query/key head h / (Hv / Hqk)
 *     (torch.repeat_interleave semantics).
 *   - Launches are asynchronous and ordered on `stream` (a cudaStream_t; NULL
 *     is the legacy default stream).  Every function is reentrant.
 *   - Return value: 0 on success, else a GDN_ERR_* code; no entry point ever
 *     aborts the process.  Failures detected on the device (a bounded wait
 *     that timed out) are OR-ed into the optional `status` word as
 *     GDN_DEVERR_* bits; the host reads it after synchronising.
 */
#ifndef GDN_B200_H
#define GDN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDN_B200_ABI_VERSION 1

typedef struct CUstream_st* gdn_stream_t; /* == cudaStream_t */

/* element types */
enum {
  GDN_DT_F32 = 0,
  GDN_DT_BF16 = 1,
  GDN_DT_F16 = 2,
};

/* how `g` encodes the forget gate */
enum {
  GDN_GATE_LOG = 0,    /* decay = exp(g)   (BASELINE / FLA convention)           */
  GDN_GATE_LINEAR = 1, /* decay = g        (the reference's `alpha` argument)    */
};

/* host-side return codes */
enum {
  GDN_OK = 0,
  GDN_ERR_NULL = 1,        /* a required pointer is NULL                        */
  GDN_ERR_SHAPE = 2,       /* unsupported or inconsistent sizes                 */
  GDN_ERR_ALIGN = 3,       /* pointer or stride breaks 16-byte alignment        */
  GDN_ERR_DTYPE = 4,       /* unsupported dtype / gate-kind combination         */
  GDN_ERR_LAUNCH = 5,      /* the CUDA launch itself failed                     */
  GDN_ERR_DEVICE = 6,      /* no device, or the device is not sm_100            */
  GDN_ERR_WORKSPACE = 7,   /* workspace missing or too small                    */
  GDN_ERR_DEVICE_WAIT = 8, /* a device-side wait timed out (from the status)    */
};

/* decode option flags (gdn_decode_args_t.flags) */
enum {
  GDN_DECODE_L2NORM_QK = 1u << 0, /* q, k <- x / sqrt(sum x^2 + l2_eps) in-kernel    */
  GDN_DECODE_GATE_RAW = 1u << 1,  /* g is the raw gate projection a:                */
                                  /*   log gate = -exp(A_log[h]) softplus(a + dt_bias[h]) */
  GDN_DECODE_OUT_NORM_GATE = 1u << 2, /* o <- RMSNorm(o) * norm_weight * silu(z) per  */
                                      /* (b, h) over d_v; needs d_v in {64, 128},    */
                                      /* d_k <= 128                                  */
};

/* device-side status bits (OR-ed into *status) */
enum {
  GDN_DEVERR_FULL_TIMEOUT = 1u << 0,  /* consumer waited too long for a slab      */
  GDN_DEVERR_EMPTY_TIMEOUT = 1u << 1, /* producer waited too long for a free slot */
  GDN_DEVERR_MMA_TIMEOUT = 1u << 2,   /* tensor-core completion never signalled   */
  GDN_DEVERR_DRAIN_TIMEOUT = 1u << 3, /* copies in flight never landed on abort   */
  GDN_DEVERR_PEER_TIMEOUT = 1u << 4,  /* a peer never released an output slot     */
};

/*
 * One decode step for a batch of sequences (GDN when g is [B,Hv], KDA when
 * g is [B,Hv,d_k]).  Strides are in ELEMENTS and cover the (batch, head)
 * axes; the innermost dimension of q/k/v/o (and of the KDA gate) must be
 * contiguous.  Element strides times the element size must be multiples of
 * 16 bytes and q/k/v/o/g base pointers 16-byte aligned (the rows are staged
 * with cp.async.bulk).
 */
typedef struct {
  const void* q;        /* [B, Hqk, d_k]   io_dtype                         */
  const void* k;        /* [B, Hqk, d_k]   io_dtype                         */
  const void* v;        /* [B, Hv,  d_v]   io_dtype                         */
  const void* g;        /* GDN: [B, Hv]; KDA: [B, Hv, d_k]   g_dtype        */
  const void* beta;     /* [B, Hv]         beta_dtype                       */
  const float* state_in;/* [B, Hv, d_k, d_v] contiguous, fp32 (or fp16, see */
                        /* state_dtype; the pointer is then reinterpreted)  */
  float* state_out;     /* same layout; may equal state_in (in place)       */
  void* o;              /* [B, Hv, d_v]    io_dtype                         */
  int64_t q_sb, q_sh, k_sb, k_sh, v_sb, v_sh, o_sb, o_sh;
  int64_t g_sb, g_sh, beta_sb, beta_sh;
  int32_t B, Hqk, Hv, dk, dv;
  int32_t io_dtype;     /* GDN_DT_BF16 or GDN_DT_F16                        */
  int32_t g_dtype;      /* any GDN_DT_*                                      */
  int32_t beta_dtype;   /* any GDN_DT_*                                      */
  int32_t gate_kind;    /* GDN_GATE_LOG or GDN_GATE_LINEAR                   */
  float scale;          /* output scale (1.0 = reference convention)         */
  uint32_t* status;     /* optional device word for GDN_DEVERR_* bits        */
  int32_t sm_reserve;   /* SMs left free for concurrent kernels (e.g. an     */
                        /* NCCL collective overlapping the step); 0 = none   */
  int32_t flags;        /* GDN_DECODE_* options (0 = none)                   */
  float l2_eps;         /* epsilon of GDN_DECODE_L2NORM_QK                   */
  const float* A_log;   /* [Hv] fp32, with GDN_DECODE_GATE_RAW (GDN only)    */
  const float* dt_bias; /* [Hv] fp32, with GDN_DECODE_GATE_RAW               */
  int32_t state_dtype;  /* GDN_DT_F32 (default) or GDN_DT_F16 (d_k = 128):   */
                        /* an fp16 state halves the bytes a step streams;    */
                        /* arithmetic stays fp32                             */
  const void* z;        /* [B, Hv, d_v] io_dtype, with GDN_DECODE_OUT_NORM_GATE */
  int64_t z_sb, z_sh;   /* element strides of z                              */
  const float* norm_weight; /* [d_v] fp32 RMSNorm weight                     */
  float norm_eps;       /* RMSNorm epsilon                                   */
  const struct gdn_peer_out* peer_out; /* optional fused output all-gather   */
                        /* over NVLink (value-head-sharded decode); NULL = none */
} gdn_decode_args_t;

/*
 * Fused output all-gather of value-head-sharded decode (one process per GPU,
 * rank r owning a contiguous range of value heads).  Every rank holds its own
 * full output buffer [B, Hv_total, d_v] (two of them, used by alternate
 * steps); `o` of the decode args points at this rank's head range inside the
 * local buffer of the step's slot (o_sb = Hv_total * d_v, o_sh = d_v), and
 * o_peer[i] at the same offset inside peer i's buffer of that slot, mapped
 * into this process (CUDA IPC).  The decode kernel stores every output row to
 * the local buffer and to each peer with plain stores over NVLink (no copy
 * engine, no collective, no TMA multicast), then:
 *   - arrival: the CTA that finishes last adds 1 to every rank's
 *     arrive[] counter (system-scope atomics after a system fence), so rank j
 *     has all outputs of step s once its counter reaches s * n_ranks;
 *   - reuse of a slot: at the start of step s this rank writes s - 1 into
 *     slot `rank` of every rank's free[] array ("I have consumed step s - 1");
 *     before its first output store of step s a CTA waits, bounded, until
 *     every entry of its own free[] is >= s - 2 (the slot's previous step was
 *     consumed everywhere).  Reads of step s's gathered outputs must therefore
 *     be ordered before this rank's next decode launch.
 * A wait that runs out sets GDN_DEVERR_PEER_TIMEOUT in the status word.
 */
typedef struct gdn_peer_out {
  void* o_peer[7];          /* peers' output bases (this rank's head offset)  */
  uint32_t* arrive[8];      /* every rank's arrival counter (self included)   */
  uint32_t* free_flags[8];  /* every rank's free[n_ranks] array               */
  uint32_t* cta_done;       /* local counter of finished CTAs (monotonic)     */
  int32_t n_ranks;          /* 2..8                                           */
  int32_t rank;             /* this rank's index                              */
  uint32_t step;            /* 1-based step number, +1 per decode launch      */
  int32_t reserved;
} gdn_peer_out_t;

/*
 * Chunked prefill over T tokens.  Tensors are contiguous [B, T, H, d]
 * (q/k: Hqk heads, v/o: Hv heads), g and beta contiguous [B, T, Hv].
 * initial_state may be NULL (zero state).  final_state receives the state
 * after token T-1.  chunk must be 64; T may be any length >= 1 (the last
 * chunk is zero-padded, which leaves state and outputs unchanged).
 * d_k = d_v = 128.  The prefill needs a device workspace of
 * gdn_prefill_workspace_size(args) bytes (16-byte aligned), owned by the
 * caller and passed in `workspace`.
 */
typedef struct {
  const void* q;            /* [B, T, Hqk, d_k] io_dtype                    */
  const void* k;            /* [B, T, Hqk, d_k] io_dtype                    */
  const void* v;            /* [B, T, Hv, d_v]  io_dtype                    */
  const void* g;            /* [B, T, Hv]       g_dtype (log gate)          */
  const void* beta;         /* [B, T, Hv]       beta_dtype                  */
  const float* initial_state; /* [B, Hv, d_k, d_v] fp32 or NULL             */
  float* final_state;       /* [B, Hv, d_k, d_v] fp32                       */
  void* o;                  /* [B, T, Hv, d_v]  io_dtype                    */
  int32_t B, T, Hqk, Hv, dk, dv, chunk;
  int32_t io_dtype, g_dtype, beta_dtype;
  float scale;
  void* workspace;          /* device scratch, >= gdn_prefill_workspace_size */
  size_t workspace_bytes;
  uint32_t* status;
} gdn_prefill_args_t;

/* Library ABI version (GDN_B200_ABI_VERSION). */
int gdn_abi_version(void);

/* Human-readable text for a GDN_ERR_* code. */
const char* gdn_status_string(int code);

/*
 * GDN decode step.  Replaces the reference's launcher
 *   launch_gdn_dispatch   (cuda-attn-gdn/attn_gdn.cu:343-358,
 *                          cuda-attn-gdn-tma/attn_gdn_tma.cu:521-545)
 * and the cuTile kernel launch ct.launch(..., gdn_decode, (Q,K,V,Alpha,Beta,
 * S_in,S_out,O)) (cutile-attn-gdn/main.py:116, 268-271), generalised to
 * GQA head counts, bf16 I/O, a log gate and an in-place state.
 */
int gdn_decode_launch(const gdn_decode_args_t* args, gdn_stream_t stream);

/*
 * KDA decode step (per-channel gate g[B,Hv,d_k]).  Replaces
 *   launch_kda_dispatch   (cuda-attn-kda/attn_kda.cu:327-345)
 * and ct.launch(..., kda_decode, (Q,K,V,G,Beta,S_in,S_out,O))
 * (cutile-attn-kda/main.py:206-269).
 */
int kda_decode_launch(const gdn_decode_args_t* args, gdn_stream_t stream);

/*
 * Reference-layout GDN decode: exactly the argument list of the reference's
 * launch_gdn_dispatch(shape, dQ, dK, dV, dA, dB, dS_in, dS_out, dO, stream)
 * (cuda-attn-gdn/attn_gdn.cu:343).  Q,K [B*H, d_k], V,O [B*H, d_v],
 * Alpha,Beta [B*H] in io_dtype (f16 in the reference), alpha used directly
 * (linear gate), S_in / S_out [B*H*d_k, d_v] fp32 (may alias).
 */
int gdn_decode_ref_launch(int32_t B, int32_t H, int32_t dk, int32_t dv,
                          const void* dQ, const void* dK, const void* dV,
                          const void* dAlpha, const void* dBeta,
                          const float* dS_in, float* dS_out, void* dO,
                          int32_t io_dtype, gdn_stream_t stream);

/*
 * Reference-layout KDA decode: the argument list of launch_kda_dispatch
 * (cuda-attn-kda/attn_kda.cu:327).  G [B*H, d_k] is a log gate in io_dtype.
 */
int kda_decode_ref_launch(int32_t B, int32_t H, int32_t dk, int32_t dv,
                          const void* dQ, const void* dK, const void* dV,
                          const void* dG, const void* dBeta,
                          const float* dS_in, float* dS_out, void* dO,
                          int32_t io_dtype, gdn_stream_t stream);

/*
 * Device scratch the prefill needs for these arguments, in bytes (0 if none).
 * The reference has no prefill; this is the new chunked path.
 */
size_t gdn_prefill_workspace_size(const gdn_prefill_args_t* args);

/*
 * GDN chunked prefill.  No reference counterpart exists (the reference only
 * describes it: analysis/wave15-attention-research/MECHANISMS.md:398-445); its
 * results are defined by T applications of the reference decode recurrence
 * (analysis/wave15-attention-architecture/reference/pytorch_reference_gdn.py:38-91).
 * The state update takes the per-token residuals beta (v - k^T S) as f16, so
 * their magnitude must stay below 65,504 (|v| up to about 1e4).
 */
int gdn_prefill_launch(const gdn_prefill_args_t* args, gdn_stream_t stream);

/*
 * GDN chunked prefill that allocates nothing.  No counterpart in the
 * reference: this entry point exists for callers of this library that
 * cannot allocate device memory themselves — for example a plugin inside a
 * host framework that owns the GPU memory pool and exposes no allocator to
 * it, or a caller that must not trigger cudaMalloc's implicit device
 * synchronisation on its serving path.  Such a caller still passes its
 * inputs and outputs (args->workspace and args->workspace_bytes are ignored);
 * the workspace gdn_prefill_launch would take lives instead in a fixed
 * device array of GDN_PREFILL_NOALLOC_SCRATCH_BYTES inside this library,
 * which every GPU that loads the library holds until the process exits.
 *   - Limit: one record of GDN_PREFILL_WS_RECORD_BYTES per (sequence, value
 *     head, 64-token chunk), i.e. B * Hv * ceil(T / 64) <= 668 (for example
 *     one sequence of 32 value heads up to T = 1344).  Larger problems return
 *     GDN_ERR_WORKSPACE without launching anything.
 *   - Set-up: the first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress, with that device current) and caches it; make
 *     that first call before any stream capture on the device.  No call
 *     allocates device memory (no cudaMalloc, cudaFree or allocating library
 *     routine).
 *   - Sharing: every call on a device uses the same array, which keeps the
 *     last call's contents (nothing in it needs to start at zero).  Calls
 *     whose kernels overlap on the GPU (two streams, or two host threads)
 *     race on it: order them on one stream or serialise them.
 * Results equal gdn_prefill_launch's on the same arguments.
 */
#define GDN_PREFILL_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
#define GDN_PREFILL_WS_RECORD_BYTES 25088u
int gdn_prefill_launch_noalloc(const gdn_prefill_args_t* args, gdn_stream_t stream);

/*
 * KDA prefill: T applications of the reference's per-channel-gate step
 * naive_recurrent_kda_step
 * (analysis/wave15-attention-architecture/reference/pytorch_reference_kda.py:42-71),
 * which the reference only runs one token at a time.  Same argument struct as
 * gdn_prefill_launch, except that g is the per-channel log gate
 * [B, T, Hv, d_k] (g_dtype) and chunk is ignored.  d_k, d_v in {64, 128, 256};
 * g 16-byte aligned, beta and the states 4-byte aligned.  initial_state may
 * equal final_state (updated in place).
 * Two forms, chosen by args->workspace:
 *   - NULL: the recurrent form (state on chip, CUDA cores), any listed d.
 *   - non-NULL (d_k = d_v = 128 only; >= kda_prefill_workspace_size bytes,
 *     16-byte aligned, as are the states): the chunked tensor-core form,
 *     64-token chunks, the per-channel decays inside the WY transform; the
 *     same f16 range condition on the residuals as gdn_prefill_launch.
 */
int kda_prefill_launch(const gdn_prefill_args_t* args, gdn_stream_t stream);

/*
 * Workspace of the chunked KDA prefill for these arguments, in bytes: one
 * 66,048-byte record per (sequence, value head, 64-token chunk), plus a
 * 16-byte count and 4 bytes per chunk for the list of chunks whose decays
 * need the slow path; 0 when the shapes have no chunked form (d_k or d_v
 * other than 128).
 */
size_t kda_prefill_workspace_size(const gdn_prefill_args_t* args);

/* ------------------------------------------------------------------------
 * Multi-GPU: all-gather of per-rank decode outputs with the copy engines.
 * The reference is single-GPU (METHODOLOGY.md:80); these entry points have no
 * counterpart there.  They serve value-head-sharded decode with one process
 * per GPU on one NVLink node.
 * ---------------------------------------------------------------------- */
#define GDN_IPC_HANDLE_BYTES 64

/* Exports a CUDA IPC handle (GDN_IPC_HANDLE_BYTES bytes) for the allocation
 * containing dev_ptr, and dev_ptr's byte offset inside that allocation. */
int gdn_ipc_handle(const void* dev_ptr, void* handle_out, uint64_t* offset_out);

/* Maps a peer process's allocation into this process (current device; peer
 * access is enabled on demand): *dev_ptr_out = mapped base + offset.  Close
 * with gdn_ipc_close(*base_out). */
int gdn_ipc_open(const void* handle, uint64_t offset, void** dev_ptr_out, void** base_out);
int gdn_ipc_close(void* base);

/* On `stream`: copy `bytes` from `src` into each peer_dst[i] (cudaMemcpyAsync,
 * a DMA over NVLink, no SMs), then write `value` into each *peer_flag[i].  The
 * flag writes are ordered after all copies on the stream. */
int gdn_gather_push(const void* src, size_t bytes, void* const* peer_dst,
                    uint32_t* const* peer_flag, int32_t n_peers, uint32_t value,
                    gdn_stream_t stream);

/* Makes `stream` wait (on the GPU front end) until flags[i] >= value for all
 * i < n. */
int gdn_gather_wait(const uint32_t* flags, int32_t n, uint32_t value, gdn_stream_t stream);

/* S_out[i] = M[i] S_in[i] + L[i] for `count` row-major fp32 d x d matrices
 * (d a multiple of 64; S_out must not alias S_in), in fp32: the start-state
 * scan of the sequence-parallel prefill, which composes the affine maps
 * S_end = M S_start + L of consecutive time segments.  No reference
 * counterpart (the reference is single-GPU). */
int gdn_state_affine(const float* M, const float* L, const float* S_in, float* S_out,
                     int32_t count, int32_t d, gdn_stream_t stream);

/* On `stream`: waits (a one-thread kernel, bounded; a timeout sets
 * GDN_DEVERR_PEER_TIMEOUT in *status) until *counter >= target, for the
 * arrival counter of the fused output all-gather (gdn_peer_out_t.arrive). */
int gdn_gather_wait_counter(const uint32_t* counter, uint32_t target, uint32_t* status,
                            gdn_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H */
