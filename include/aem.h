/*
 * aem.h -- C ABI of the B200 (sm_100a) MoE-layer hot path of AetherMoE.
 *
 * Plain C: pointers, sizes and opaque handles only.  Every call returns an
 * aem_status; on failure aem_last_error() holds a thread-local message.  No
 * C++ exception crosses this boundary.
 *
 * Pointer conventions:
 *   *_host functions take host pointers and copy through the context's
 *   pinned staging buffers; every other compute call takes DEVICE pointers
 *   and runs asynchronously on the given stream (a cudaStream_t passed as
 *   void*; NULL = the legacy default stream).  Packed weight handles are
 *   immutable after creation and may be shared between threads and streams.
 *
 * Layout conventions follow the reference Python API (the src/kernels modules):
 *   hidden [N, D] row-major, gate_weight [D, E], gate_bias [E],
 *   q_int8 [D, E] (= [K, N]) with per-output-column scale [1, E].
 */
#ifndef AEM_H
#define AEM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status, dtypes, limits ------------------------------------------------ */

typedef enum {
    AEM_OK = 0,
    AEM_EINVAL = 1,       /* bad argument: shape, limit, null pointer (reference: ValueError) */
    AEM_ECUDA = 2,        /* a CUDA runtime/driver call failed */
    AEM_ENCCL = 3,        /* an NCCL call failed */
    AEM_ETIMEOUT = 4,     /* a bounded device or host wait gave up */
    AEM_ENOMEM = 5,       /* device or pinned-host allocation failed */
    AEM_EUNSUPPORTED = 6, /* no sm_100 device, or the build lacks the feature */
    AEM_EDEVICE = 7       /* a kernel reported a failed in-kernel check (e.g. bad batch_position) */
} aem_status;

typedef enum { AEM_F32 = 0, AEM_BF16 = 1 } aem_dtype;

/* Gating logit arithmetic.
 * EXACT: each product is a float32 product and products are summed in
 *   float32 in increasing d order, bias last -- bit-identical logits to the
 *   reference's fused_kernel_simulation (prototype/math_proto.py:19-50), so
 *   indices match it bit-exactly on every row.
 * FAST: fused multiply-adds (one rounding per term) in the same order;
 *   indices match on every row whose k-th/(k+1)-th logit gap exceeds
 *   float32 rounding.
 * CERTIFIED: indices bit-identical to EXACT on every row, at FAST speed or
 *   better: logits are computed with fused multiply-adds (for small batches
 *   with d split over threads) beside a rigorous bound on their distance
 *   from the EXACT logits (per 64-wide block of d: the partial sums'
 *   magnitudes and Cauchy-Schwarz bounds of sum |x w|); a row whose selected
 *   experts' bound intervals are ordered and clear of every other expert's
 *   is certified and written from the fast logits (values within float32
 *   rounding of EXACT's); every other row -- near ties, NaN, +-inf -- is
 *   recomputed with the EXACT arithmetic (written exactly as EXACT writes it)
 *   on the device, without a host round trip.  aem_gate_fallback_rows counts
 *   the recomputed rows.  CERTIFIED calls on one gate share that gate's
 *   device list of deferred rows: they must not overlap on the GPU (issue
 *   them on one stream, or one gate per stream). */
typedef enum {
    AEM_GATING_EXACT = 0,
    AEM_GATING_FAST = 1,
    AEM_GATING_CERTIFIED = 2
} aem_gating_mode;

#define AEM_MAX_EXPERTS 256 /* fused_gating_metal.py:230 MAX_EXPERTS */
#define AEM_MAX_TOPK 64     /* fused_gating_metal.py:231 MAX_TOPK */
#define AEM_CAPACITY_UNLIMITED UINT64_MAX /* router.hpp:50 RouterConfig default */

/* Thread-local message of the last failing call on this thread ("" if none). */
const char* aem_last_error(void);
/* Library version string. */
const char* aem_version(void);
/* Number of sm_100 devices visible (0 on a host without a B200). */
int aem_device_count(void);
/* Synchronises `stream` and reports (then clears) the in-kernel check and
 * bounded-wait failures the library's kernels recorded on the current
 * device since the last check: AEM_OK, AEM_EDEVICE or AEM_ETIMEOUT. */
aem_status aem_device_status(void* stream);

/* Total number of kernels this library has launched in this process (all
 * devices, all entry points): lets a caller count the launches of a step. */
uint64_t aem_kernel_launches(void);

/* Phases of a layer step whose device time can be profiled. */
enum {
    AEM_PHASE_GATING = 0,   /* fused gating */
    AEM_PHASE_ROUTE = 1,    /* capacity routing, permutation, row gather */
    AEM_PHASE_UP = 2,       /* grouped INT8 up GEMM + ReLU */
    AEM_PHASE_DOWN = 3,     /* grouped INT8 down GEMM */
    AEM_PHASE_COMBINE = 4,  /* weighted combine */
    AEM_PHASE_DISPATCH = 5, /* expert parallel: token rows to expert owners */
    AEM_PHASE_RETURN = 6,   /* expert parallel: expert outputs back */
    AEM_PHASE_EXCHANGE = 7, /* expert parallel: count all-gathers and the size sync */
    AEM_NUM_PHASES = 8
};

/* ---- host-side context (staging for *_host calls) ------------------------- */

typedef struct aem_context_s* aem_context_t;
/* Creates a context bound to `device`: one stream, grow-only pinned host and
 * device staging buffers.  Not thread-safe: use one context per thread. */
aem_status aem_context_create(int device, aem_context_t* out);
aem_status aem_context_destroy(aem_context_t ctx);
/* The context's stream (cudaStream_t as void*). */
void* aem_context_stream(aem_context_t ctx);

/* ---- fused gating ------------------------------------------------------------ */

typedef struct aem_gate_s* aem_gate_t;

/* Packs a gating layer: gate_weight [D, E] and gate_bias [E] float32 from
 * HOST memory into a device-resident copy laid out [ceil(D/4)][Epad][4]
 * (Epad = E rounded up to 8..256): every 4 consecutive d of one expert are one
 * 16-byte vector, and one chunk of d is contiguous for all experts.
 * Replaces _get_transposed_weight, src/kernels/fused_gating_metal.py:328-344
 * (the cached [E, D] transpose), with caller-owned lifetime.
 * gate_bias may be NULL (zero bias).  E <= AEM_MAX_EXPERTS. */
aem_status aem_gate_pack(const float* gate_weight, const float* gate_bias, int64_t D, int64_t E,
                         int device, aem_gate_t* out);
aem_status aem_gate_free(aem_gate_t gate);
/* Rows of this gate's CERTIFIED-mode calls that were recomputed with the
 * EXACT arithmetic (not certified), since the gate was packed; synchronises
 * the gate's device.  No counterpart in the reference. */
aem_status aem_gate_fallback_rows(aem_gate_t gate, int64_t* rows);

/* Fused gating: logits = hidden @ gate_weight + gate_bias, top-k by repeated
 * strict-greater max extraction (ties -> lowest expert id), softmax over the
 * k selected logits.  Replaces the kernel launch of fused_gating,
 * src/kernels/fused_gating_metal.py:361-435 (MSL body :236-307).
 * Non-finite logits select as np.argmax in the reference's specification
 * (prototype/math_proto.py:38-42): NaN ranks above every number (the first
 * NaN first), and a winner is overwritten with -inf rather than removed, so
 * a row with fewer than k + k_extra logits above -inf repeats its lowest
 * -inf id; every written id is in [0, E).
 *   hidden   device [N, D], dtype AEM_F32 or AEM_BF16
 *   out_idx  device int32 [N, k + k_extra]: descending-logit expert ids; the
 *            k_extra (0 or 1) trailing id is the next choice (the capacity
 *            reroute target) and gets no weight.  k + k_extra <= E.
 *   out_val  device float32 [N, k]: softmax weights (row sums to 1).
 * Errors as the reference (ValueError -> AEM_EINVAL): k > AEM_MAX_TOPK, k > E,
 * k < 1.  N == 0 is a no-op. */
aem_status aem_gating(aem_gate_t gate, const void* hidden, aem_dtype hidden_dtype, int64_t N,
                      int k, int k_extra, aem_gating_mode mode, int32_t* out_idx, float* out_val,
                      void* stream);

/* Same with HOST buffers (copies in and out through ctx; synchronous).
 * This is the call the reference-facing Python shim makes. */
aem_status aem_gating_host(aem_context_t ctx, aem_gate_t gate, const void* hidden,
                           aem_dtype hidden_dtype, int64_t N, int k, int k_extra,
                           aem_gating_mode mode, int32_t* out_idx, float* out_val);

/* ---- INT8 weight-only quantisation and GEMM ---------------------------------- */

/* Per-output-column symmetric INT8 quantisation, bit-exact with float32
 * NumPy: scale[n] = max(max_k |w[k,n]| / 127, 1e-12); q = clip(rint(w/scale),
 * -127, 127).  Device pointers: w f32 [K, N], q int8 [K, N], scale f32 [N].
 * Replaces quantize_weights, src/kernels/quantized_gemm.py:70-76
 * (prototype/math_proto.py:52-66). */
aem_status aem_quantize_int8(const float* w, int64_t K, int64_t N, int8_t* q, float* scale,
                             void* stream);
/* HOST-buffer form of aem_quantize_int8 (synchronous). */
aem_status aem_quantize_int8_host(aem_context_t ctx, const float* w, int64_t K, int64_t N,
                                  int8_t* q, float* scale);

typedef struct aem_qweight_s* aem_qweight_t;

/* Packs G groups (experts) of INT8 weights from HOST memory:
 * q [G][K][N] int8 (reference layout) and scale [G][N] float32 become a
 * device-resident copy tiled for the GEMM's weight stream (every block of
 * 128 output channels x 64 K is one contiguous 8 KB tile).
 * Replaces _get_transposed_qweight, src/kernels/quantized_gemm.py:151-167.
 * The tensor-core path needs K % 8 == 0 (16-byte activation rows); other K
 * use a CUDA-core kernel. */
aem_status aem_qweight_pack(const int8_t* q, const float* scale, int64_t G, int64_t K, int64_t N,
                            int device, aem_qweight_t* out);
/* Same from DEVICE memory (q [G][K][N], scale [G][N]); stream-ordered. */
aem_status aem_qweight_pack_device(const int8_t* q, const float* scale, int64_t G, int64_t K,
                                   int64_t N, void* stream, aem_qweight_t* out);
aem_status aem_qweight_free(aem_qweight_t w);
/* Dimensions of a packed weight (any pointer may be NULL). */
aem_status aem_qweight_shape(aem_qweight_t w, int64_t* G, int64_t* K, int64_t* N);

/* out[M, N] (float32) = x[M, K] @ (q[group] * scale[group]).  Dequantises
 * at multiply time: int8 tiles are converted to bf16 in shared memory and
 * multiplied on the tcgen05 tensor cores with float32 accumulation in TMEM;
 * float32 x is split into two bf16 terms (hi + lo).  Device pointers.
 * Replaces fused_quantized_matmul, src/kernels/quantized_gemm.py:184-226
 * (MSL body :99-138).  D mismatch -> AEM_EINVAL as the reference (:202-205). */
aem_status aem_qgemm(aem_qweight_t w, int64_t group, const void* x, aem_dtype x_dtype, int64_t M,
                     float* out, void* stream);
/* Grouped form (the per-expert GEMM of an MoE layer): activation rows
 * [group_rows[g], group_rows[g+1]) (device int32 array of G+1 offsets) are
 * multiplied by weight group g of `w` (G <= 256, G <= groups of w):
 *   out[rowmap ? rowmap[r] : r][n] (=|+=) act(rowscale[r] * scale[g][n] * sum_k x[r,k] q[g][n,k])
 * x bf16 [M, K] (device); out float32 or bf16 with row stride ldo; act = ReLU
 * when relu != 0; accumulate != 0 adds with float32 red.add (out must be
 * float32; rows may repeat); rowmap/rowscale may be NULL.  token_tile is
 * the rows per tile (16, 32, 64, 128, 256; 0 = chosen from M/G) and ksplit
 * splits K across CTAs (needs accumulate).  No counterpart call in the
 * reference: its kernels take one weight matrix per call. */
aem_status aem_grouped_qgemm(aem_qweight_t w, const int32_t* group_rows, int G, const void* x,
                             int64_t M, void* out, aem_dtype out_dtype, int64_t ldo, int relu,
                             int accumulate, const int32_t* rowmap, const float* rowscale,
                             int token_tile, int ksplit, void* stream);
/* Which form of the tensor-core GEMM runs (process-wide, every device):
 * -1 (default) automatic -- token tiles of 128 or 256 rows over an even
 * number of 128-channel blocks (or at least 11) run on SM pairs (tcgen05
 * cta_group::2: two SMs share one 256-channel tile, each holding half of
 * the token rows), everything else on single SMs; 0 single SMs only; 1 SM
 * pairs from 64-row tiles on.  Results agree within float32 summation
 * order.  No counterpart in the reference. */
aem_status aem_set_gemm_pairs(int mode);
/* Where the tensor-core GEMM keeps the converted bf16 weights (process-wide):
 * -1 (default) automatic -- tensor memory (the MMA reads A from TMEM, so
 * shared memory carries only the int8 stream and the activations) for token
 * tiles up to 64 rows, shared memory above; 0 shared memory only; 1 tensor
 * memory for every tile (token tiles capped at 192 rows, no SM pairs, and
 * also for the few-row calls that otherwise take the weight-stream kernel).
 * Results agree within float32 summation order.  No counterpart in the
 * reference. */
aem_status aem_set_gemm_tmem_a(int mode);
/* HOST-buffer form of aem_qgemm (synchronous). */
aem_status aem_qgemm_host(aem_context_t ctx, aem_qweight_t w, int64_t group, const void* x,
                          aem_dtype x_dtype, int64_t M, float* out);

/* ---- capacity-ceiling routing -------------------------------------------------- */

/* Effective expert of each of n tokens: within each primary-expert group,
 * ranked by batch_position, the first `capacity` keep their primary and the
 * rest take their own secondary (one hop).  Replaces
 * Router::assign_effective_experts, src/orchestration/router.hpp:249-266.
 * Device pointers, uint32 [n].  batch_position must be a permutation of
 * [0, n) (the reference's reassembly rejects anything else,
 * router.hpp:286-313); a violation returns AEM_EDEVICE.  Expert ids < E.
 * capacity = AEM_CAPACITY_UNLIMITED keeps every primary.
 * workspace: device scratch of aem_capacity_route_workspace(n, E) bytes, or
 * NULL to have the call allocate (stream-ordered) and free it.  The call
 * synchronises the stream to report in-kernel check failures. */
size_t aem_capacity_route_workspace(int64_t n, int E);
aem_status aem_capacity_route(const uint32_t* primary, const uint32_t* secondary,
                              const uint32_t* batch_position, int64_t n, int E, uint64_t capacity,
                              uint32_t* effective, void* workspace, size_t workspace_bytes,
                              void* stream);

/* Capacity routing that allocates no device memory.  No counterpart in the
 * reference: it exists for callers that cannot call cudaMalloc while they
 * run -- a serving loop that reserves its whole device budget at start-up
 * and may not grow it, or one that cannot pay the device-wide
 * synchronisation cudaFree implies in the middle of a step.  Same rule,
 * arguments and results as aem_capacity_route, but the scratch is a fixed
 * array of AEM_ROUTE_STATIC_SCRATCH_BYTES in the library's device memory,
 * held on every GPU that loads the library until the process exits.
 *   - n > AEM_ROUTE_STATIC_MAX_UNITS (or E > AEM_MAX_EXPERTS) -> AEM_EINVAL.
 *   - Every call looks the array's address up on the current device (a
 *     lookup that allocates nothing; the first one on a device loads the
 *     library's device code there), so a cudaDeviceReset between calls is
 *     safe; make the first call on a device before any stream capture.
 *   - Every call on a device shares the one array and it keeps the last
 *     call's contents (each call resets what must start at zero): calls
 *     that overlap on the GPU -- on different streams or from different
 *     host threads -- race.  Serialise them.
 *   - It synchronises `stream` to report in-kernel check failures. */
#define AEM_ROUTE_STATIC_MAX_UNITS 262144
#define AEM_ROUTE_STATIC_SCRATCH_BYTES 4325632
aem_status aem_capacity_route_static(const uint32_t* primary, const uint32_t* secondary,
                                     const uint32_t* batch_position, int64_t n, int E,
                                     uint64_t capacity, uint32_t* effective, void* stream);

/* ---- MoE layer (gating -> routing -> grouped INT8 expert FFN -> combine) --------- */

typedef struct {
    int64_t d_model;       /* hidden size d */
    int64_t d_ffn;         /* expert FFN size */
    int num_experts;       /* E (global) */
    int top_k;             /* k */
    uint64_t capacity;     /* per-expert capacity per step, or AEM_CAPACITY_UNLIMITED */
    aem_gating_mode gating_mode;
} aem_moe_config;

typedef struct aem_moe_s* aem_moe_t;

/* A single-GPU MoE layer.  `up` holds E groups of [d_model -> d_ffn]
 * (q [E][d_model][d_ffn]), `down` E groups of [d_ffn -> d_model].  The
 * handles are borrowed and must outlive the layer. */
aem_status aem_moe_create(const aem_moe_config* cfg, aem_gate_t gate, aem_qweight_t up,
                          aem_qweight_t down, aem_moe_t* out);
aem_status aem_moe_free(aem_moe_t moe);

/* One layer step on device buffers: x [T, d] (F32/BF16) -> out [T, d]
 * (F32/BF16).  Units are the (token, slot) pairs in slot-major order
 * (batch_position = j*T + t); a unit's secondary is the token's (k+1)-th
 * gating choice; capacity is applied as Router::assign_effective_experts
 * (router.hpp:249-266); each unit runs relu(x W_up) W_down of its effective
 * expert and out[t] = sum_j weight[t,j] * y[t,j].
 * Precision (the int8 weights are exact in bf16; every product is summed in
 * float32; gating always reads x in its own dtype):
 *   x AEM_F32  -- x enters the up GEMM as a bf16 pair hi + lo (x to about 16
 *                 significant bits, two MMAs per K step) and, by default,
 *                 so does the hidden activation relu(x W_up) in the down
 *                 GEMM: the float32-activation contract of
 *                 fused_quantized_matmul (quantized_gemm.py:184-226).
 *   x AEM_BF16 -- x is used as is; the hidden activation is stored as bf16
 *                 (one MMA per K step) unless aem_moe_set_hidden_dtype
 *                 selects the pair.
 * out AEM_BF16 rounds the float32 layer output once at the end. */
aem_status aem_moe_forward(aem_moe_t moe, const void* x, aem_dtype x_dtype, int64_t T, void* out,
                           aem_dtype out_dtype, void* stream);
/* Storage of the hidden activation relu(x W_up) between the expert GEMMs:
 * -1 (default) follows x's dtype, AEM_F32 keeps it as a bf16 pair hi + lo
 * (about 16 significant bits; the down GEMM then issues two MMAs per K
 * step), AEM_BF16 rounds it to bf16.  No counterpart in the reference, whose
 * kernels never compose an FFN. */
aem_status aem_moe_set_hidden_dtype(aem_moe_t moe, int hidden_dtype);
/* HOST-buffer form of aem_moe_forward (synchronous). */
aem_status aem_moe_forward_host(aem_context_t ctx, aem_moe_t moe, const void* x, aem_dtype x_dtype,
                                int64_t T, void* out, aem_dtype out_dtype);
/* Asynchronous form of aem_moe_forward_host for a stream of steps: copies x
 * in on the context's upload stream, computes on the context's stream once
 * the copy landed, copies the output out on its download stream -- so with
 * page-locked host buffers the next step's upload and the previous step's
 * download overlap the current step's compute.  Returns at once with a
 * ticket; at most three steps are in flight per context (a fourth submit
 * waits on the host for the oldest to finish): a caller that waits for step
 * i - 2 after submitting step i keeps the compute stream busy while step
 * i + 1 uploads and step i - 1 downloads.  x and out must stay valid and
 * untouched until aem_context_wait(ctx, ticket) returns, which also reports
 * the step's in-kernel errors.  Steps run in submission order. */
aem_status aem_moe_submit_host(aem_context_t ctx, aem_moe_t moe, const void* x, aem_dtype x_dtype,
                               int64_t T, void* out, aem_dtype out_dtype, uint64_t* ticket);
/* Waits for the step of `ticket` (from a *_submit_host call on ctx): its
 * output is in the host buffer when this returns AEM_OK. */
aem_status aem_context_wait(aem_context_t ctx, uint64_t ticket);
/* Per-phase profiling with CUDA events recorded on the step's stream.
 * enable != 0 starts (and clears) accumulation; aem_moe_profile_read
 * synchronises, then writes the summed milliseconds of each phase
 * (ms[AEM_NUM_PHASES]) and the number of profiled steps. */
aem_status aem_moe_profile(aem_moe_t moe, int enable);
aem_status aem_moe_profile_read(aem_moe_t moe, double* ms, int64_t* steps);
/* Routing of the last forward (device pointers, stream-ordered copies):
 * idx int32 [T, k+1] (k+1 clipped to E), val f32 [T, k], effective uint32 [T*k]. */
aem_status aem_moe_last_routing(aem_moe_t moe, int32_t* idx, float* val, uint32_t* effective,
                                void* stream);

/* ---- expert parallelism over NCCL ---------------------------------------------------- */

/* Host-side planning of the distributed capacity rule (no GPU needed).
 * counts: [R][k][E] per-rank primary counts per (slot, expert).  Writes
 * base [k][E] for `rank`: the global rank offset of this rank's first unit
 * in each (slot, expert) group, with units ordered slot-major by global
 * batch_position and tokens split contiguously over ranks. */
aem_status aem_ep_plan_bases(const int64_t* counts, int R, int k, int E, int rank, int64_t* base);

/* Host-side planning of one expert-parallel exchange (no GPU needed).
 * starts: [R][E+1] every rank's first expert-grouped row per expert (the
 * all-gathered output of the routing step).  For `rank`, writes the
 * contiguous send segment to each peer p (send_off/send_cnt[p], rows of its
 * expert-grouped buffer holding experts p*E/R .. (p+1)*E/R-1), the receive
 * segment from each peer (recv_off/recv_cnt[p], peers in rank order), and
 * groups [R*E/R + 1]: row offsets of the received (peer, local expert)
 * segments -- the grouped GEMM's row groups. */
aem_status aem_ep_plan_exchange(const int32_t* starts, int R, int E, int rank, int64_t* send_off,
                                int64_t* send_cnt, int64_t* recv_off, int64_t* recv_cnt,
                                int32_t* groups);

/* Largest expert-parallel world (ranks that map each other's memory). */
#define AEM_EP_MAX_RANKS 64

/* Where one rank's rows go in the peer-memory exchange of one step.  Units
 * are (token, slot) rows; pairs are (token, destination rank) rows -- a
 * token's activation crosses NVLink once per destination rank, and the
 * destination returns one pre-reduced float32 row per pair.  Every rank's
 * tokens are split in two halves (A = the first ceil(T/2), B = the rest) that
 * travel and compute as a two-stage pipeline: a destination holds its half-A
 * units first, then its half-B units, each expert-major with sources in rank
 * order inside; a source's pairs for one destination list half-A tokens
 * first. */
typedef struct aem_ep_peer_plan {
    int32_t ok;         /* 1 when every rank's segments fit the receive capacities */
    int32_t units_in;   /* units this rank receives, both halves */
    int32_t units_in_a; /* of which half A (rows [0, units_in_a)) */
    int32_t pairs_in;   /* pairs this rank receives */
    int32_t pairs_out;  /* pairs this rank sends (rows of its return buffer) */
    int32_t dst_unit_off[2][AEM_MAX_EXPERTS]; /* [half][expert position]: this rank's first
                                                 unit row of that expert in its owner's buffer */
    int32_t dst_pair_off[AEM_EP_MAX_RANKS];      /* this rank's first pair row in rank r's buffer */
    int32_t send_pair_off[AEM_EP_MAX_RANKS];     /* this rank's pairs for rank r start here */
    int32_t send_pair_a[AEM_EP_MAX_RANKS];       /* ... of which the first send_pair_a are half A */
    int32_t recv_pair_off[AEM_EP_MAX_RANKS + 1]; /* pairs received from source s start here */
    int32_t recv_pair_a[AEM_EP_MAX_RANKS];       /* ... of which the first recv_pair_a are half A */
    int32_t ret_off[AEM_EP_MAX_RANKS];           /* row in s's return buffer of s's first pair here */
} aem_ep_peer_plan;

/* Host form of the per-step plan the expert-parallel layer computes on the
 * device (no GPU needed).  all: [R][AEM_EP_PAYLOAD(E, R)] int32, every rank's
 * payload: expert starts [E+1] (units grouped by expert position, half A
 * first inside each expert), pair counts per destination [R], its live mask
 * [2] (not read here), half-A units per expert [E], half-A pairs per
 * destination [R].  live: bit r set when rank r takes part in the step; the
 * rows of other ranks are ignored, and so are units for them (those units
 * fail).  Capacities: units_cap (received units), pairs_cap (received
 * pairs), ret_cap (return rows), the same on every rank.  Writes the plan of
 * `rank` and groups [2][E/R+1]: for each half, the row offsets of the received
 * units of each local expert (half B's offsets continue after half A's).  A
 * plan whose counts do not fit or do not add up has ok = 0 (every rank
 * derives the same verdict from the same data). */
#define AEM_EP_PAYLOAD(E, R) ((((E) * 2 + 3 + (R) * 2) + 3) & ~3)
aem_status aem_ep_plan_peer(const int32_t* all, int R, int E, int rank, uint64_t live,
                            int64_t units_cap, int64_t pairs_cap, int64_t ret_cap,
                            aem_ep_peer_plan* plan, int32_t* groups);
/* The same plan computed by the layer's device code (one thread block, in
 * parallel over ranks and experts) on DEVICE buffers, asynchronously on
 * `stream`: lets a caller check the device plan against aem_ep_plan_peer. */
aem_status aem_ep_plan_peer_device(const int32_t* all, int R, int E, int rank, uint64_t live,
                                   int64_t units_cap, int64_t pairs_cap, int64_t ret_cap,
                                   aem_ep_peer_plan* plan, int32_t* groups, void* stream);

/* NCCL unique id (128 bytes) for aem_ep_create; made on one rank and
 * broadcast by the caller. */
aem_status aem_ep_unique_id(uint8_t out[128]);

typedef struct aem_ep_s* aem_ep_t;

/* One rank of an expert-parallel MoE layer: E/R experts per rank, placed by
 * expert_to_rank [E] (the reference Router's expert_to_shard,
 * router.hpp:55-60; NULL = contiguous blocks, e / (E/R), the map of
 * tests/test_orchestration.cpp:25-33).  `up_local`/`down_local` hold this
 * rank's experts in increasing expert id.  Routing does not depend on the
 * placement (bit-exact either way); load balance does.  Replaces the
 * Router + ICollectiveTransport scatter/gather (router.hpp:67-100,
 * collective_transport.hpp:37-51): activations and expert outputs move by
 * stores into the peers' memory over NVLink (CUDA IPC, mapped once here),
 * and so do the step's small all-gathers and barriers (flags with a
 * deadline); NCCL only bootstraps the mapping here and tears it down in
 * aem_ep_free.  Every rank must run on its own GPU.  Collective:
 * every rank calls it with the same config and max_tokens_local, the most
 * tokens any rank passes to one aem_ep_forward (receive buffers are sized
 * for the worst case, so a step never allocates). */
aem_status aem_ep_create(const aem_moe_config* cfg, int rank, int world, const uint8_t uid[128],
                         aem_gate_t gate, aem_qweight_t up_local, aem_qweight_t down_local,
                         const int32_t* expert_to_rank, int64_t max_tokens_local, aem_ep_t* out);
aem_status aem_ep_free(aem_ep_t ep);
/* One step: this rank's T_local tokens (global positions rank*T_local ...)
 * -> its outputs.  Precision: activations cross NVLink and enter the expert
 * GEMMs as bf16 -- float32 x is rounded to bf16 once, at dispatch -- and the
 * hidden activation is stored as bf16; products are summed in float32 and
 * outputs are float32 sums (the single-GPU layer's bf16 mode).  Collective: every rank calls it with the same T_local
 * (<= max_tokens_local).  Asynchronous on `stream` (no host synchronisation);
 * a receive-capacity or peer failure is reported by aem_device_status
 * (AEM_ETIMEOUT for a silent peer), the way route_batch throws. */
aem_status aem_ep_forward(aem_ep_t ep, const void* x, aem_dtype x_dtype, int64_t T_local, void* out,
                          aem_dtype out_dtype, void* stream);
/* Tolerant step: Router::route_batch_tolerant (router.hpp:127-234).  Never
 * reports a peer failure as an error: every (token, slot) unit gets exactly
 * one outcome, unit_failed[j*T_local + t] = 0 (its expert output is in
 * out[t]) or 1 (it contributes nothing).  A unit fails when its effective
 * expert lives on a rank marked unhealthy, or when the step itself fails
 * because a peer did not signal within the deadline (every unit of the step
 * then fails, on every rank that took part, and out is zero).  A rank that
 * timed out is remembered as unhealthy by aem_ep_health and left out of later
 * steps, like the Router's unhealthy_shards_ (no reconnection).
 * unit_failed: device uint8 [k*T_local] (slot-major) or NULL. */
aem_status aem_ep_forward_tolerant(aem_ep_t ep, const void* x, aem_dtype x_dtype, int64_t T_local,
                                   void* out, aem_dtype out_dtype, uint8_t* unit_failed,
                                   void* stream);
/* HOST-buffer form of aem_ep_forward: copies x in and out through ctx (whose
 * device must be this rank's) and synchronises; collective like
 * aem_ep_forward.  A peer failure is returned as AEM_ETIMEOUT / AEM_EDEVICE. */
aem_status aem_ep_forward_host(aem_context_t ctx, aem_ep_t ep, const void* x, aem_dtype x_dtype,
                               int64_t T_local, void* out, aem_dtype out_dtype);
/* Asynchronous form of aem_ep_forward_host (see aem_moe_submit_host):
 * collective -- every rank submits the same sequence of steps. */
aem_status aem_ep_submit_host(aem_context_t ctx, aem_ep_t ep, const void* x, aem_dtype x_dtype,
                              int64_t T_local, void* out, aem_dtype out_dtype, uint64_t* ticket);
/* The host learned that `rank` is gone (a store, a heartbeat, a process
 * exit): later steps leave it out and never touch its memory again.  A rank
 * that exited must be marked here before the next step; the in-step deadline
 * covers a rank that stops taking part but keeps its process. */
aem_status aem_ep_mark_unhealthy(aem_ep_t ep, int rank);
/* Synchronises `stream`, folds the ranks the device found silent into the
 * unhealthy set and writes that set (bit r = rank r) to *unhealthy.
 * Router::is_shard_unhealthy / unhealthy_shard_count (router.hpp:236-240). */
aem_status aem_ep_health(aem_ep_t ep, uint64_t* unhealthy, void* stream);
/* Two-half pipeline of a step (half B's dispatch under half A's GEMMs, half
 * A's return under half B's): mode -1 = automatic (currently off: measured
 * slower at 2 and 4 ranks), 0 = off, 1 = on.  Collective: every rank must use
 * the same mode. */
aem_status aem_ep_set_pipeline(aem_ep_t ep, int mode);
/* Deadline of every in-step wait on a peer (default 2 s). */
aem_status aem_ep_set_timeout(aem_ep_t ep, double seconds);
/* Per-phase profiling of this rank's steps (see aem_moe_profile). */
aem_status aem_ep_profile(aem_ep_t ep, int enable);
aem_status aem_ep_profile_read(aem_ep_t ep, double* ms, int64_t* steps);
/* Routing of the last step for this rank's units (device pointers):
 * idx [T_local, k+1], val [T_local, k], effective [k*T_local] (slot-major). */
aem_status aem_ep_last_routing(aem_ep_t ep, int32_t* idx, float* val, uint32_t* effective,
                               void* stream);

/* ---- scheduler -> MoE layer seam ----------------------------------------------------- */

/* One sequence's share of a continuous-batching iteration: the reference's
 * StepResult (src/core/scheduler.hpp:43-48) plus where that sequence's rows
 * live -- `tokens` consecutive hidden rows (a prefill chunk, or 1 for a
 * decode step). */
typedef struct aem_seq_slice {
    uint64_t seq_id;
    const void* x; /* device [tokens, d_model], x dtype */
    void* out;     /* device [tokens, d_model], out dtype */
    int64_t tokens;
} aem_seq_slice;

/* Runs one ContinuousBatchingScheduler::step() iteration
 * (src/core/scheduler.hpp:75-146) through the MoE layer as ONE batch, in the
 * order of `slices` (the scheduler's result order: decode steps, then prefill
 * chunks): batch_position follows that order, so capacity routing ranks the
 * iteration's tokens exactly as over their concatenation.  One kernel gathers
 * the slices' rows, aem_moe_forward runs, one kernel scatters the outputs.
 * No counterpart in the reference, which never connects its scheduler to the
 * kernels (README.md:392-397).  Slices with tokens == 0 are allowed. */
aem_status aem_moe_forward_slices(aem_moe_t moe, const aem_seq_slice* slices, int n_slices,
                                  aem_dtype x_dtype, aem_dtype out_dtype, void* stream);

/* ---- per-step telemetry ---------------------------------------------------------- */

/* The reference's TelemetryRecorder / TelemetryFlusher pattern
 * (src/core/telemetry.hpp:131-250) for MoE-layer steps: a process-wide
 * switch (default off; one relaxed atomic load per step when off); when on,
 * every aem_moe_forward / aem_ep_forward(_tolerant) records its device time
 * with a CUDA event pair on its stream, harvested without ever waiting on an
 * unfinished step. */
enum { AEM_METRIC_MOE_STEP = 0, AEM_METRIC_EP_STEP = 1, AEM_NUM_METRICS = 2 };
typedef struct aem_metric_stats {
    uint64_t count; /* MetricStats (telemetry.hpp:35-42): nearest-rank percentiles */
    double mean_ns, p50_ns, p95_ns, p99_ns, max_ns;
} aem_metric_stats;
void aem_telemetry_enable(int enabled); /* TelemetryRecorder::set_enabled */
int aem_telemetry_enabled(void);
/* Statistics of every completed step of `metric` so far
 * (TelemetryFlusher::snapshot); *dropped (nullable) = steps not recorded
 * because too many were in flight or the sample store was full. */
aem_status aem_telemetry_snapshot(int metric, aem_metric_stats* out, uint64_t* dropped);
aem_status aem_telemetry_reset(void); /* TelemetryRecorder::reset_for_testing */
/* The snapshot's arithmetic on given latencies (host, no GPU):
 * detail::compute_stats, telemetry.hpp:88-113. */
aem_status aem_metric_stats_of(const uint64_t* latencies_ns, int64_t n, aem_metric_stats* out);

#ifdef __cplusplus
}
#endif

#endif /* AEM_H */
