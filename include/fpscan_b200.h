/*
 * fpscan_b200 — C ABI of the B200 (sm_100a) linear-recurrence scan library.
 *
 *     y[t] = gates[t] * y[t-1] + tokens[t],   y[-1] = 0,
 * along the last axis of contiguous (batch, dim, seqlen) tensors.
 *
 * Conventions for every entry point:
 *   - All pointers are device pointers of the CURRENT CUDA device, 16-byte
 *     aligned; tensors are row-major (rows = batch*dim rows of `seqlen`
 *     elements).  Element type is given by `dtype` (FPSCAN_F32/F16/BF16);
 *     per-row carry buffers are always fp32.
 *   - Work is enqueued asynchronously on `stream` (a cudaStream_t; NULL is
 *     the legacy default stream).  No scan, backward or shard call
 *     allocates device memory (scratch comes from caller workspaces or
 *     fixed arrays inside the library); the only allocation is the chained
 *     mode's mailbox, made once by fpscan_link_create.  Calls are
 *     re-entrant.  Every kernel is launched with programmatic dependent
 *     launch: its prologue overlaps the previous kernel in the stream, and
 *     it touches global memory only after that kernel completed.  The
 *     streaming kernels hand rows to
 *     their CTAs through a counter word that each launch takes from a fixed
 *     array in the library's own device memory (zero between launches), so
 *     launches on different streams may run concurrently, and a launch
 *     recorded into a CUDA graph keeps its word for every replay.  Make the
 *     first call on a device outside any stream capture; launches captured
 *     before it use static row tiles (same results, bit for bit).
 *   - Return 0 on success.  Non-zero: FPSCAN_ERR_INVALID (bad argument,
 *     nothing launched) or FPSCAN_ERR_CUDA (launch failed); the message is in
 *     fpscan_last_error() of the calling thread.
 *   - Arithmetic is fp32 for every storage type.
 */
#ifndef FPSCAN_B200_H
#define FPSCAN_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FPSCAN_OK 0
#define FPSCAN_ERR_INVALID 1
#define FPSCAN_ERR_CUDA 2

#define FPSCAN_F32 0
#define FPSCAN_F16 1
#define FPSCAN_BF16 2

#define FPSCAN_ABI_VERSION 1

#if defined(__GNUC__)
#define FPSCAN_API __attribute__((visibility("default")))
#else
#define FPSCAN_API
#endif

/* Version of this ABI (FPSCAN_ABI_VERSION). */
FPSCAN_API int fpscan_abi_version(void);

/*
 * Forward or reverse scan, zero initial state; the gate of the first element
 * in scan order is ignored.  `out` may be exactly `tokens` or `gates`
 * (in place); any other overlap is rejected.  seqlen: power of two in
 * [32, 65536].
 * Replaces fpscan._C.fullscan_forward(gates, tokens, out, reverse)
 * (reference csrc/main.cpp:10 -> warpscan_fwd, csrc/full_scan/full_scan.h:26-36,
 * warpscan_forward, csrc/full_scan/full_scan.cu:238-258).
 */
FPSCAN_API int fpscan_scan_fwd(const void* gates, const void* tokens, void* out, int64_t batch,
                    int64_t dim, int64_t seqlen, int dtype, int reverse, void* stream);

/*
 * Bytes of workspace fpscan_scan_fwd_ws needs for this shape (0: none; the
 * shape is then served by the fpscan_scan_fwd kernel).  Non-zero when
 * batch*dim is too small to fill the GPU with one CTA per row, so rows are
 * split across CTAs.  Depends on the current device (its SM count).
 * No reference counterpart (the reference runs one CTA per row,
 * csrc/full_scan/full_scan.cu:190).
 */
FPSCAN_API int64_t fpscan_scan_fwd_workspace_bytes(int64_t batch, int64_t dim, int64_t seqlen,
                                                   int dtype);

/*
 * fpscan_scan_fwd with a caller-provided device workspace (16-byte aligned,
 * at least fpscan_scan_fwd_workspace_bytes; may be NULL when that is 0).
 * Zero the workspace once after allocating it; afterwards it can be reused by
 * any number of calls that are ordered on the GPU (e.g. one stream).
 * Calls that overlap on the GPU must use different workspaces.
 * Same results and contract as fpscan_scan_fwd (which it replaces for
 * few-channel, long-sequence shapes).
 */
FPSCAN_API int fpscan_scan_fwd_ws(const void* gates, const void* tokens, void* out,
                                  int64_t batch, int64_t dim, int64_t seqlen, int dtype,
                                  int reverse, void* workspace, int64_t workspace_bytes,
                                  void* stream);

/* Gate activations for the *_act entry points: the kernels read
 * pre-activation values z and use gates = act(z) (computed in fp32). */
#define FPSCAN_ACT_NONE 0
#define FPSCAN_ACT_SIGMOID 1           /* gates = 1 / (1 + exp(-z))            */
#define FPSCAN_ACT_EXP_NEG_SOFTPLUS 2  /* gates = exp(-softplus(z)) = 1/(1+e^z) */
#define FPSCAN_ACT_EXP 3               /* gates = exp(z)                        */

/*
 * fpscan_scan_fwd on gates = act(z): the activation that produces the gates
 * (e.g. sigmoid, or BASELINE config 4's exp(-softplus(z))) is applied as the
 * chunk is loaded, so the separate elementwise pass over z (read z, write
 * gates) disappears.  No reference counterpart (extends fullscan_forward).
 */
FPSCAN_API int fpscan_scan_fwd_act(const void* z, const void* tokens, void* out, int64_t batch,
                                   int64_t dim, int64_t seqlen, int dtype, int reverse,
                                   int activation, void* stream);

/*
 * fpscan_scan_bwd for y = scan(act(z), tokens): writes dz = dgates * act'(z)
 * instead of dgates (the producer's backward fused in), and dtokens.
 * No reference counterpart.
 */
FPSCAN_API int fpscan_scan_bwd_act(const void* z, const void* y, const void* grad_out, void* dz,
                                   void* dtokens, int64_t batch, int64_t dim, int64_t seqlen,
                                   int dtype, int activation, void* stream);

/*
 * fpscan_scan_fwd for ANY seqlen >= 1.  The reference accepts only powers of
 * two in [32, 65536] (csrc/full_scan/full_scan.cu:207-233, README.md:101-106);
 * this entry point has no counterpart there and lifts that limit (masked row
 * tails; rows need not start on a 16-byte boundary, only the three base
 * pointers must be 16-byte aligned).  Zero initial state, `out` may equal
 * `gates` or `tokens`, otherwise as fpscan_scan_fwd.
 */
FPSCAN_API int fpscan_scan_fwd_anylen(const void* gates, const void* tokens, void* out,
                                      int64_t batch, int64_t dim, int64_t seqlen, int dtype,
                                      int reverse, void* stream);

/*
 * fpscan_scan_bwd (the fused PScan.backward, fpscan/ops.py:70-83) for any
 * seqlen >= 1.  No reference counterpart.  Outputs must not overlap inputs.
 */
FPSCAN_API int fpscan_scan_bwd_anylen(const void* gates, const void* y, const void* grad_out,
                                      void* dgates, void* dtokens, int64_t batch, int64_t dim,
                                      int64_t seqlen, int dtype, void* stream);

/*
 * Channel-last layout: gates, tokens, out are (batch, seqlen, dim) contiguous
 * and the recurrence runs along seqlen: y[b,t,d] = gates[b,t,d]*y[b,t-1,d] +
 * tokens[b,t,d], zero initial state (reverse: from t = seqlen-1).  The
 * reference has no such layout: its README (README.md:94-99) transposes with
 * .mT.contiguous() around pscan.  Any seqlen >= 1; dim*itemsize must be a
 * multiple of 16.  Needs a workspace of fpscan_cl_workspace_bytes() bytes
 * (16-byte aligned; 256 bytes when batch*ceil(dim_vectors/8) >= 128, else
 * the per-segment maps of the few-column path: columns x segments x
 * channels x 12 bytes, well under a megabyte for such shapes; calls that may
 * overlap need separate workspaces).  `out` may equal gates or tokens.
 */
FPSCAN_API int64_t fpscan_cl_workspace_bytes(int64_t batch, int64_t seqlen, int64_t dim,
                                             int dtype, int backward);
FPSCAN_API int fpscan_scan_fwd_cl(const void* gates, const void* tokens, void* out,
                                  int64_t batch, int64_t seqlen, int64_t dim, int dtype,
                                  int reverse, void* workspace, int64_t workspace_bytes,
                                  void* stream);

/*
 * Fused backward (fpscan/ops.py:70-83 semantics) in the channel-last layout:
 * dtokens[t] = grad_out[t] + gates[t+1]*dtokens[t+1], dgates[t] =
 * dtokens[t]*y[t-1], along seqlen.  Outputs must not overlap anything.
 */
FPSCAN_API int fpscan_scan_bwd_cl(const void* gates, const void* y, const void* grad_out,
                                  void* dgates, void* dtokens, int64_t batch, int64_t seqlen,
                                  int64_t dim, int dtype, void* workspace,
                                  int64_t workspace_bytes, void* stream);

/*
 * Scan with a per-row initial state `init` (fp32, batch*dim values):
 * y[0] = gates[0]*init + tokens[0] (reverse: y[L-1] = gates[L-1]*init +
 * tokens[L-1]).  The final state is the last element of out in scan order.
 * Otherwise as fpscan_scan_fwd.  Extends the reference, whose initial state
 * is fixed at zero (csrc/full_scan/full_scan.cu:96).
 */
FPSCAN_API int fpscan_scan_fwd_init(const void* gates, const void* tokens, void* out,
                                    const float* init, int64_t batch, int64_t dim,
                                    int64_t seqlen, int dtype, int reverse, void* stream);

/*
 * fpscan_scan_fwd for callers that cannot allocate device memory (a host
 * that owns every GPU allocation, a service that forbids cudaMalloc/cudaFree
 * while running, C code without a caching allocator).  Same arguments and
 * results as fpscan_scan_fwd / fpscan_scan_fwd_ws; the scratch that
 * few-channel, long-sequence shapes need comes from a fixed array inside the
 * library (8,448 bytes per GPU, held until exit: at most 512 split
 * segments; larger needs are rejected with FPSCAN_ERR_INVALID).  Whether a
 * shape needs split segments, and how many, depends on the GPU's SM count
 * and occupancy (fpscan_scan_fwd_workspace_bytes gives the need: the call
 * accepts the shape when that is at most 8,448).  The first call on a device
 * looks the array's address up (make it before any stream capture).  Every
 * call clears the array's tile counter on its own stream.  Calls share the
 * array: calls that overlap on the GPU race and must not be issued.
 * Allocates nothing.
 * No counterpart in the reference.
 */
FPSCAN_API int fpscan_scan_fwd_noalloc(const void* gates, const void* tokens, void* out,
                                       int64_t batch, int64_t dim, int64_t seqlen, int dtype,
                                       int reverse, void* stream);

/*
 * Fused backward of y = scan(gates, tokens):
 *   dtokens[t] = gates[t+1]*dtokens[t+1] + grad_out[t]  (last element: grad_out)
 *   dgates[t]  = dtokens[t] * y[t-1]                      (first element: 0*dtokens)
 * One launch, reads gates/y/grad_out once, writes dgates/dtokens.  Outputs
 * must not overlap any input or each other.  seqlen as fpscan_scan_fwd.
 * Replaces the composition in PScan.backward (reference fpscan/ops.py:70-83:
 * two torch.cat shifts, a reverse fullscan_forward and a multiply).
 */
FPSCAN_API int fpscan_scan_bwd(const void* gates, const void* y, const void* grad_out, void* dgates,
                    void* dtokens, int64_t batch, int64_t dim, int64_t seqlen, int dtype,
                    void* stream);

/*
 * fpscan_scan_bwd for few, long rows: rows are cut into segments processed
 * by separate CTAs with a decoupled look-back on the dtokens state (the
 * split-row scheme of fpscan_scan_fwd_ws, run from each row's end).
 * `workspace` (16-byte aligned; zero it once after allocating it, as for
 * fpscan_scan_fwd_ws) of at least fpscan_scan_bwd_workspace_bytes(...)
 * bytes; that query returns 0 for
 * shapes the split-row path does not take, and then this call is
 * fpscan_scan_bwd.  Outputs must not overlap any input, each other or the
 * workspace.  Calls sharing one workspace must be ordered (one stream).
 * Extends fpscan_scan_bwd, which replaces the composition in
 * PScan.backward (reference fpscan/ops.py:70-83).
 */
FPSCAN_API int64_t fpscan_scan_bwd_workspace_bytes(int64_t batch, int64_t dim, int64_t seqlen,
                                                   int dtype);
FPSCAN_API int fpscan_scan_bwd_ws(const void* gates, const void* y, const void* grad_out,
                                  void* dgates, void* dtokens, int64_t batch, int64_t dim,
                                  int64_t seqlen, int dtype, void* workspace,
                                  int64_t workspace_bytes, void* stream);

/* ---- Sequence-sharded building blocks (no reference counterpart: the
 * reference has no multi-GPU path).  A shard holds `rows` rows of `seqlen`
 * (power of two, >= 32, <= 2^24) consecutive positions of longer sequences. */

/* Per row: carry_a = product of all gates, carry_b = scan's last value with
 * zero initial state.  Reads gates and tokens, writes 2 floats per row. */
FPSCAN_API int fpscan_shard_fwd_reduce(const void* gates, const void* tokens, float* carry_a,
                            float* carry_b, int64_t rows, int64_t seqlen, int dtype,
                            void* stream);

/* Forward scan with per-row initial state y_init (y[0] = gates[0]*y_init + tokens[0]). */
FPSCAN_API int fpscan_shard_fwd_scan(const void* gates, const void* tokens, void* out,
                          const float* y_init, int64_t rows, int64_t seqlen, int dtype,
                          void* stream);

/* Per row: carry_b = gates[0] * dtokens[0], dtokens computed with zero value
 * entering from the right.  Reads gates and grad_out. */
FPSCAN_API int fpscan_shard_bwd_reduce(const void* gates, const void* grad_out, float* carry_b,
                            int64_t rows, int64_t seqlen, int dtype, void* stream);

/* Fused backward of a shard: `addend` (per row) enters at the last element
 * (dtokens[L-1] = addend + grad_out[L-1]); `y_prev` (per row) is y just
 * before the shard's first element, used for dgates[0]. */
FPSCAN_API int fpscan_shard_bwd_scan(const void* gates, const void* y, const void* grad_out,
                          void* dgates, void* dtokens, const float* addend,
                          const float* y_prev, int64_t rows, int64_t seqlen, int dtype,
                          void* stream);

/* Fold gathered per-shard maps.  `gathered` is fp32 [world][2][rows]
 * (A then B).  reverse=0: out = compose shards 0..rank-1 applied to 0;
 * reverse=1: compose shards world-1..rank+1.  out: fp32 [rows]. */
FPSCAN_API int fpscan_carry_combine(const float* gathered, int world, int rank, int64_t rows,
                         int reverse, float* out, void* stream);

/*
 * Chained sequence sharding over NVLink peer memory (no reference
 * counterpart; the reference has no multi-GPU path).  Rank r holds positions
 * [r*L/world, (r+1)*L/world) of every row; instead of reduce + all-gather +
 * scan (fpscan_shard_*), each rank's scan waits for the state entering each
 * row from rank r-1 and hands the row's final state to rank r+1 (backward:
 * the reverse direction) through a per-rank "mailbox" that the neighbours
 * map with CUDA IPC.  Ranks must be distinct GPUs of one node.  Every wait is
 * bounded (2 s, then status bit 3 is set and 0 is used).
 *
 * fpscan_link_bytes / _create / _destroy: the mailbox (cudaMalloc'd once,
 * zeroed; `depth` ring slots per direction, epochs counted per direction
 * starting at 1, slot = epoch % depth).  _ipc_handle writes 64 bytes to
 * share with the neighbours; _open / _close map / unmap a neighbour's.
 */
FPSCAN_API int64_t fpscan_link_bytes(int64_t rows, int depth);
FPSCAN_API int fpscan_link_create(int64_t rows, int depth, void** mailbox);
FPSCAN_API int fpscan_link_destroy(void* mailbox);
FPSCAN_API int fpscan_link_ipc_handle(void* mailbox, void* handle);
FPSCAN_API int fpscan_link_open(const void* handle, void** peer_mailbox);
FPSCAN_API int fpscan_link_close(void* peer_mailbox);

/*
 * Forward scan of this rank's shard (rows x seqlen, local seqlen a power of
 * two larger than one chunk): zero initial state on the first rank (prev ==
 * NULL), otherwise the state from rank r-1 (also stored to init_record when
 * it is not NULL: the backward needs it); each row's final state goes to
 * rank r+1 unless next == NULL.
 */
FPSCAN_API int fpscan_shard_fwd_link(const void* gates, const void* tokens, void* out,
                                     float* init_record, int64_t rows, int64_t seqlen, int dtype,
                                     void* local, void* prev, void* next, uint32_t epoch,
                                     int depth, void* stream);

/*
 * Fused backward of this rank's shard: the value entering each row's last
 * element comes from rank r+1 (next != NULL), gates[0]*dtokens[0] of each
 * row goes to rank r-1 (prev != NULL); y_prev = the forward's init_record
 * (y of the previous shard's last element; NULL on the first rank).
 */
FPSCAN_API int fpscan_shard_bwd_link(const void* gates, const void* y, const void* grad_out,
                                     void* dgates, void* dtokens, const float* y_prev,
                                     int64_t rows, int64_t seqlen, int dtype, void* local,
                                     void* prev, void* next, uint32_t epoch, int depth,
                                     void* stream);

/* Message of the last failed call on this thread ("" if none). */
FPSCAN_API const char* fpscan_last_error(void);

/* Synchronously read (and if `clear`, reset) the current device's status
 * word.  Bit 0: a kernel gave up a bounded wait on its own copies; bit 1: a
 * split-row scan gave up waiting for a preceding segment; bit 2: a
 * channel-last CTA found its shared-memory staging buffer misaligned for TMA
 * and skipped its work; bit 3: a chained sequence-sharded scan gave up
 * waiting for a neighbouring rank (fpscan_shard_*_link); bit 4 (16, only in
 * the bounds-checking build): a kernel skipped a global access outside its
 * tensor.  Results of such a launch are not valid.  0 = healthy. */
FPSCAN_API int fpscan_device_status(unsigned* status, int clear);

/* Enqueue on `stream` a read-and-clear of the current device's status word
 * into *dst (4 bytes of device memory, or of pinned host memory mapped into
 * the device's address space), without synchronising: a caller checks the
 * value once the stream has reached it (an event), so failures of a launch
 * can be raised without stalling the host.  Allocates nothing.  The
 * reference has no device-side waits and no counterpart. */
FPSCAN_API int fpscan_status_snapshot(unsigned* dst, void* stream);

/* Set the limit of every bounded device-side wait (copies landing, split-row
 * look-back, chained neighbour ranks) on the current device, in ns, within
 * [1 ms, 600 s]; default 2 s.  A wait that runs out sets its status bit and
 * returns: a look-back or a neighbour value that never came is replaced by
 * NaN, so the affected rows are visibly wrong.  Synchronous (a copy to a
 * device symbol); set it while no scan runs.  No counterpart in the
 * reference. */
FPSCAN_API int fpscan_set_wait_limit_ns(uint64_t ns);

/* Test hook of the bounds-checking build (libfpscan_b200_debug.so, built
 * with -DFPSCAN_DEBUG_BOUNDS: every global access a kernel computes is
 * checked against its tensor's extent; one outside is skipped and sets
 * status bit 4).  Returns 1 in that build, 0 in the release build, -1 on a
 * launch error, after enqueueing on `stream` a probe kernel that, in the
 * bounds-checking build only, checks (without accessing it) an address just
 * past an extent -- so that build's status word shows bit 4 afterwards.
 * No counterpart in the reference. */
FPSCAN_API int fpscan_debug_bounds(void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FPSCAN_B200_H */
