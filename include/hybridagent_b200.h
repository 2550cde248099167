/*
 * hybridagent_b200.h -- C ABI of the B200 (sm_100a) ZeRO-1 AdamW step.
 *
 * Drop-in boundary for HybridAgent's ZeroOneAdamW (hybrid_rl/optimizer.py).  The
 * reference has no native code; its optimizer calls torch eager ops and
 * torch.distributed.  Each entry point below names the reference lines it replaces.
 * The Python class hybridagent_b200.ZeroOneAdamW binds these through ctypes; any
 * other host language binds the same symbols.
 *
 * Conventions
 *   - Every function returns HA_OK (0) or an HA_ERR_* code; ha_last_error() gives the
 *     calling thread's last message.
 *   - Device addresses are plain pointers (or uint64_t inside tables); `stream` is a
 *     cudaStream_t passed as void*.  Nothing here synchronizes the stream unless stated.
 *   - Tables marked "device" live in device memory the caller owns; tables marked
 *     "host" are read before the call returns.
 *   - Rounding follows torch's CUDA elementwise kernels op by op, so results equal the
 *     reference optimizer run on a CUDA device bit for bit (fp32 state and the
 *     low-precision parameter copy); see the per-function notes.
 */
#ifndef HYBRIDAGENT_B200_H_
#define HYBRIDAGENT_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HA_OK 0
#define HA_ERR_INVALID 1     /* bad argument or table entry */
#define HA_ERR_CUDA 2        /* CUDA runtime error (message carries cudaGetErrorString) */
#define HA_ERR_NCCL 3        /* NCCL error */
#define HA_ERR_UNSUPPORTED 4 /* dtype combination or feature not built */

/* element types */
#define HA_F32 0
#define HA_BF16 1
#define HA_F16 2
#define HA_F64 3
#define HA_I32 4
#define HA_U8 5

/* Elements per chunk of the multi-tensor kernels: one CTA processes one chunk. */
#define HA_ADAMW_CHUNK 16384
#define HA_SUMSQ_CHUNK 32768
#define HA_SUM_REGIONS_CHUNK 16384

/* Largest number of peers a rank can push to (an NVLink domain of 16 GPUs). */
#define HA_MAX_PEERS 15
#define HA_IPC_HANDLE_BYTES 64

const char* ha_last_error(void);
int ha_abi_version(void);

/* ------------------------------------------------------------------ tables */

/* One owned tensor of the update (device table, 64 bytes).
 * Mirrors the per-tensor state of optimizer.py:57-76 and the per-step scalars of
 * optimizer.py:180-189.  grad == 0 means "no gradient" (optimizer.py:174: skipped,
 * no decay, no step).  param == 0 means the fp32 master is the parameter itself
 * (fp32 parameters, optimizer.py:71-73). */
typedef struct ha_tensor {
  uint64_t grad;       /* gradient, dtype grad_dtype of the launch */
  uint64_t master;     /* fp32 */
  uint64_t exp_avg;    /* fp32 */
  uint64_t exp_avg_sq; /* fp32 */
  uint64_t param;      /* param_dtype copy written as round-to-nearest-even of master */
  int64_t numel;
  float decay;         /* (float)(1 - lr*weight_decay)          optimizer.py:185 */
  float neg_lr;        /* (float)(-lr)                          optimizer.py:189 */
  float rc1;           /* (float)(1.0 / (1 - beta1**step))      optimizer.py:182,189 */
  float rc2;           /* (float)(1.0 / (1 - beta2**step))      optimizer.py:183,188 */
} ha_tensor;

/* One chunk: elements [index*chunk, min((index+1)*chunk, numel)) of table entry `tensor`. */
typedef struct ha_chunk {
  uint32_t tensor;
  uint32_t index;
} ha_chunk;

/* One entry of a multi-tensor copy (device table, 32 bytes): numel elements of
 * elem_bytes each from src to dst; src == 0 writes zeros; src == dst is skipped. */
typedef struct ha_copy {
  uint64_t src;
  uint64_t dst;
  int64_t numel;
  int64_t reserved;
} ha_copy;

/* Per-launch scalars of the update (host struct, passed by pointer). */
typedef struct ha_adamw_scalars {
  float b1;        /* (float)beta1                 optimizer.py:186 */
  float a1;        /* (float)(1 - beta1) */
  float b2;        /* (float)beta2                 optimizer.py:187 */
  float a2;        /* (float)(1 - beta2) */
  float eps;       /* (float)eps                   optimizer.py:188 */
  int32_t use_decay; /* weight_decay != 0          optimizer.py:184 */
  int32_t clip;      /* 1: gradients are scaled by clip_mult first (optimizer.py:155-159) */
  float clip_mult;   /* fp32 multiplier torch applies for grad.mul_(scale) in grad_dtype */
} ha_adamw_scalars;

/* ------------------------------------------------------------------ host helpers (no GPU needed) */

/* Greedy largest-first ownership, ties to the lowest rank, equal sizes in list order
 * (replaces optimizer.py:46-53).  owner_out[n]. */
int ha_greedy_owners(int64_t n, const int64_t* numels, int32_t world, int32_t* owner_out);

/* Chunk list of the tensors with include[i] != 0 (include == NULL: all), in table
 * order.  Writes at most `cap` chunks; *n_out is the number needed. */
int ha_plan_chunks(int64_t n_tensors, const int64_t* numels, const uint8_t* include, int64_t chunk_elems,
                   ha_chunk* out, int64_t cap, int64_t* n_out);

/* Checks a chunk list against tensor sizes (host copies): every tensor index in range,
 * every chunk start inside its tensor. */
int ha_check_chunks(int64_t n_tensors, const int64_t* numels, const ha_chunk* chunks, int64_t n_chunks,
                    int64_t chunk_elems);

/* Fills decay / neg_lr / rc1 / rc2 of n host table entries from each tensor's lr and
 * step count, in double exactly as optimizer.py:180-185 computes them, then cast to
 * fp32 (corrections through libm pow, as CPython's float ** does). */
int ha_fill_step_scalars(int64_t n, const double* lrs, const int64_t* steps, double beta1, double beta2,
                         double weight_decay, ha_tensor* table);

/* Per-launch scalars (optimizer.py:186-188) and the clip multiplier: torch's mul_ of a
 * bf16 / fp16 / fp32 gradient by a Python scale multiplies float(g) by (float)scale and
 * rounds the product to the gradient's dtype (optimizer.py:159). */
int ha_make_scalars(double beta1, double beta2, double eps, double weight_decay, int grad_dtype, int clip,
                    double clip_scale, ha_adamw_scalars* out);

/* ------------------------------------------------------------------ device kernels */

/* Fused multi-tensor AdamW (replaces optimizer.py:173-191, the per-tensor loop of about
 * thirteen eager kernels): per element reads grad, master, exp_avg, exp_avg_sq once,
 * writes master, exp_avg, exp_avg_sq and the param copy once (28 bytes for bf16
 * grad/param).  grad_dtype and param_dtype are HA_F32 / HA_BF16 / HA_F16 for every
 * entry of the launch; param_dtype is ignored for entries whose param == 0.
 * chunk_elems must be HA_ADAMW_CHUNK. */
int ha_adamw_step(const ha_tensor* d_tensors, const ha_chunk* d_chunks, int64_t n_chunks, int64_t chunk_elems,
                  int grad_dtype, int param_dtype, const ha_adamw_scalars* scalars, void* stream);

/* Sum of float(g)**2 over the gradients of the listed chunks (replaces the per-tensor
 * grad.float().square().sum() of optimizer.py:149-151).  d_partials[n_chunks] receives one
 * fp64 partial per chunk; d_out[0] receives their sum in a fixed order, so the result
 * does not depend on scheduling.  Entries with grad == 0 contribute nothing.
 * chunk_elems must be HA_SUMSQ_CHUNK. */
int ha_grad_sumsq(const ha_tensor* d_tensors, const ha_chunk* d_chunks, int64_t n_chunks, int64_t chunk_elems,
                  int grad_dtype, double* d_partials, double* d_out, void* stream);

/* ha_grad_sumsq on at most max_ctas CTAs (0: one per chunk, as ha_grad_sumsq), each taking
 * every max_ctas-th chunk.  For a sum launched beside other kernels (the square sums taken
 * while backward still runs, at world size 1), which a capped grid leaves most SMs to.  The
 * partials and the result are the same, bit for bit, for every max_ctas.  No counterpart in
 * the reference. */
int ha_grad_sumsq_ctas(const ha_tensor* d_tensors, const ha_chunk* d_chunks, int64_t n_chunks, int64_t chunk_elems,
                       int grad_dtype, double* d_partials, double* d_out, int max_ctas, void* stream);

/* Allocation-free ha_grad_sumsq, for callers that cannot allocate device scratch (an
 * engine whose pools already hold nearly all of HBM, a loop that must avoid the implicit
 * synchronization of cudaMalloc / cudaFree, a host binding without a device allocator).
 * No counterpart in the reference.  The per-chunk partials live in a fixed array inside
 * the library, reserved on every GPU that loads it until exit; n_chunks above
 * HA_NOALLOC_SUMSQ_MAX_CHUNKS is rejected with HA_ERR_INVALID.  The first call on a device
 * looks up that array's device address (with the device current) and caches it; make
 * that first call before any stream capture.  All calls share the array: calls whose
 * kernels overlap on the GPU race.  Same result as ha_grad_sumsq, bit for bit. */
#define HA_NOALLOC_SUMSQ_MAX_CHUNKS 262144
int ha_grad_sumsq_noalloc(const ha_tensor* d_tensors, const ha_chunk* d_chunks, int64_t n_chunks,
                          int64_t chunk_elems, int grad_dtype, double* d_out, void* stream);

/* In-place grad.mul_(scale) over the listed chunks, rounding to grad_dtype
 * (optimizer.py:157-159); mult is ha_adamw_scalars.clip_mult. */
int ha_scale_grads(const ha_tensor* d_tensors, const ha_chunk* d_chunks, int64_t n_chunks, int64_t chunk_elems,
                   int grad_dtype, float mult, void* stream);

/* Multi-tensor copy / zero-fill (replaces the bucket packing of optimizer.py:126-135).
 * chunk_elems elements of elem_bytes (2 or 4) per chunk.  Destinations may be peer-mapped
 * memory (the p2p gradient push). */
int ha_gather(const ha_copy* d_copies, const ha_chunk* d_chunks, int64_t n_chunks, int64_t chunk_elems,
              int elem_bytes, void* stream);

/* ha_gather on at most max_ctas (> 0) CTAs that walk the chunk list with the grid's stride:
 * the early gradient pushes made while backward still runs (gradient landing at
 * hybrid_rl/train.py:268's loss.backward()) occupy a few SMs instead of all of them. */
int ha_gather_capped(const ha_copy* d_copies, const ha_chunk* d_chunks, int64_t n_chunks, int64_t chunk_elems,
                     int elem_bytes, int32_t max_ctas, void* stream);

/* The same copies from a HOST table, issued to the copy engines: one cudaMemcpyAsync
 * (src != 0) or cudaMemsetAsync (src == 0, zero-fill) per entry on `stream`; entries with
 * src == dst are skipped.  Uses no SM. */
int ha_copy_async(const ha_copy* h_copies, int64_t n, int elem_bytes, void* stream);


/* ------------------------------------------------------------------ peer-to-peer (NVLink / NVSwitch) */

/* Byte offsets from this rank's packed parameter buffer to every peer's mapping of that
 * peer's packed parameter buffer (same layout on all ranks). */
typedef struct ha_peers {
  int32_t n;                    /* number of peers (world - 1), at most HA_MAX_PEERS */
  int32_t reserved;
  int64_t delta[HA_MAX_PEERS];  /* peer address = local address + delta[q] */
} ha_peers;

/* Device memory that can be shared with other processes through CUDA IPC (the packed
 * parameter and gradient-receive buffers of world > 1). */
int ha_malloc(size_t bytes, void** out);
int ha_free(void* ptr);
int ha_memset(void* ptr, int value, size_t bytes, void* stream);
int ha_ipc_get_handle(const void* ptr, uint8_t out[HA_IPC_HANDLE_BYTES]);
int ha_ipc_open(const uint8_t handle[HA_IPC_HANDLE_BYTES], void** out);
int ha_ipc_close(void* ptr);

/* Owner side of the gradient reduction (replaces the dist.reduce of optimizer.py:136 and
 * the norm's square-sum of :149-151 in one pass): d_regions holds `world` regions of
 * region_elems elements, region r written by rank r's push (ha_gather into the owner's
 * receive buffer).  Elements [0, count) of all regions are added in fp32 in rank order
 * 0..world-1, rounded once to dtype and written to d_sum[0, count) (which may alias one
 * region); the sum of squares of the written values goes to d_partials (one per
 * HA_SUM_REGIONS_CHUNK) and d_out[0].  At world 2 this equals any SUM reduction of the two
 * gradients bit for bit. */
int ha_sum_regions(const void* d_regions, int32_t world, int64_t region_elems, int64_t count, void* d_sum, int dtype,
                   double* d_partials, double* d_out, void* stream);

/* ha_adamw_step that also stores every updated parameter value (the low-precision copy,
 * or the fp32 master when the master is the parameter) at the same offset in each peer's
 * packed parameter buffer: the parameter all-gather of optimizer.py:192-194 fused into the
 * update.  The caller orders the peers' next reads after a collective. */
int ha_adamw_step_peers(const ha_tensor* d_tensors, const ha_chunk* d_chunks, int64_t n_chunks,
                        int64_t chunk_elems, int grad_dtype, int param_dtype, const ha_adamw_scalars* scalars,
                        const ha_peers* peers, void* stream);

/* ha_adamw_step for 16-bit parameters (param_dtype HA_BF16 or HA_F16, the gradient of the
 * same type) that stores a 4-element group of the parameter copy only where its rounded value
 * changes -- the `param.copy_(master.to(param.dtype))` of optimizer.py:191 -- and, with
 * `peers` non-NULL, stores those groups also into every peer's packed parameter buffer (the
 * broadcast of optimizer.py:192-194).  The caller guarantees that on entry every copy of each
 * parameter (local and peers') equals RNE(master); the result is then bit for bit that of a
 * full write on every copy, while unchanged groups cost no HBM write and no NVLink bytes.
 * A changed group is stored with the other groups of its 32-byte sector (whole sectors, no
 * read-modify-write).  d_changed_groups (device, may be NULL): the number of groups stored
 * (elements of the scalar paths count one each) is added to it. */
int ha_adamw_step_delta(const ha_tensor* d_tensors, const ha_chunk* d_chunks, int64_t n_chunks, int64_t chunk_elems,
                        int param_dtype, const ha_adamw_scalars* sc, const ha_peers* peers,
                        unsigned long long* d_changed_groups, void* stream);

/* ------------------------------------------------------------------ NCCL (NVLink / NVSwitch) */

typedef struct ha_comm ha_comm;

/* 128-byte NCCL unique id, created on one rank and handed to all (e.g. over the
 * caller's process group). */
int ha_comm_unique_id(uint8_t out[128]);
/* Communicator on the calling thread's current CUDA device. */
int ha_comm_init(const uint8_t id[128], int32_t world, int32_t rank, ha_comm** out);
int ha_comm_destroy(ha_comm* comm);
/* Aborts the communicator (ncclCommAbort): collectives blocked on a rank that stopped
 * answering end, and every later call on it returns HA_ERR_NCCL.  Safe from a watchdog
 * thread while the caller waits on the stream; the caller must not enqueue concurrently.
 * The reference relies on the process group's timeout for this (hybrid_rl/dist.py:29). */
int ha_comm_abort(ha_comm* comm);

/* SUM reduce-scatter: recv[count] = sum over ranks of send[rank*count .. +count]
 * (replaces the per-owner bucketed dist.reduce of optimizer.py:108-142). In place when
 * recv == send + rank*count*elem_bytes. */
int ha_reduce_scatter(ha_comm* comm, const void* send, void* recv, size_t count, int dtype, void* stream);
/* All-gather: recv[r*count ..] = send of rank r (replaces the per-tensor
 * dist.broadcast of optimizer.py:192-194).  In place when send == recv + rank*count. */
int ha_all_gather(ha_comm* comm, const void* send, void* recv, size_t count, int dtype, void* stream);
/* SUM all-reduce in place (optimizer.py:153 for the norm). */
int ha_all_reduce_sum(ha_comm* comm, void* buf, size_t count, int dtype, void* stream);
/* MAX all-reduce in place (optimizer.py:105 for the used mask). */
int ha_all_reduce_max(ha_comm* comm, void* buf, size_t count, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HYBRIDAGENT_B200_H_ */
