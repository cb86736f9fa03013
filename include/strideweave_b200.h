/*
 * strideweave_b200.h - C ABI of the B200 CUDA carrier for StrideWeave.
 *
 * Every entry point is `extern "C"`, takes plain pointers and sizes, returns an
 * `int` status (SW_OK on success) and never aborts.  On failure the calling
 * thread's message is available from sw_last_error().  Device pointers are
 * addresses returned by sw_alloc (or any cudaMalloc'd address); `stream` is a
 * cudaStream_t passed as `void*` (NULL = the legacy default stream).  Kernel
 * entry points only enqueue work: they return before the device has finished.
 *
 * The reference (patrickk1998/strideweave) binds its CPU kernels through
 * pybind11; these functions are what its Python carrier layer reaches through
 * ctypes instead.  Each declaration names the reference interface it replaces.
 */
#ifndef STRIDEWEAVE_B200_H
#define STRIDEWEAVE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Everything declared here is exported from the shared library even when it
 * is built with hidden default visibility. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ---- status codes ------------------------------------------------------- */
#define SW_OK 0
#define SW_ERR_INVALID 1     /* bad argument: shape, stride, dtype, alignment  */
#define SW_ERR_UNSUPPORTED 2 /* a valid request no kernel implements           */
#define SW_ERR_CUDA 3        /* a CUDA runtime/driver call failed              */
#define SW_ERR_TIMEOUT 4     /* a bounded device-side wait gave up             */
#define SW_ERR_NOMEM 5       /* device allocation failed                       */

/* ---- limits ------------------------------------------------------------- */
#define SW_MAX_LEAVES 8   /* leaves per top-level mode in a strided plan */
#define SW_MAX_SWIZZLE 4  /* XOR stages of a carrier-level swizzle       */

/* ---- runtime ------------------------------------------------------------ */

/* Message of the last failing call on this thread ("" if none). */
const char* sw_last_error(void);

/* ABI version, bumped on any incompatible change of this header. */
int sw_abi_version(void);

int sw_device_count(int* count);
int sw_set_device(int device);
int sw_get_device(int* device);

/* Device storage of a carrier's flat index space, from the device's stream-ordered
 * memory pool in the order of the legacy default stream (allocation and release
 * never synchronise the device; memory is reused without returning to the driver).
 * Replaces the owned storage of CPU(size, ...) in
 * src/strideweave/carriers/cpu/native/_cpu_carrier.hpp:38-67. */
int sw_alloc(void** ptr, int64_t bytes);
int sw_free(void* ptr);

/* Copies.  Host pointers may be pageable or pinned; pinned ones overlap. */
int sw_memcpy_h2d(void* dst, const void* src, int64_t bytes, void* stream);
int sw_memcpy_d2h(void* dst, const void* src, int64_t bytes, void* stream);
/* Device-to-host copy that returns once the copy is enqueued: with a pinned
 * destination it overlaps work on other streams; the caller synchronises the
 * stream (or an event recorded after it) before reading the destination.
 * sw_memcpy_d2h above waits for its copy.  Replaces, with sw_memcpy_h2d, the
 * host-side reads of a carrier (CPU carrier element access,
 * src/strideweave/carriers/cpu/native/_cpu_carrier.hpp:38-67). */
int sw_memcpy_d2h_async(void* dst, const void* src, int64_t bytes, void* stream);
int sw_memcpy_d2d(void* dst, const void* src, int64_t bytes, void* stream);
int sw_memset(void* dst, int value, int64_t bytes, void* stream);

/* Page-locked host buffers for overlapped host<->device copies. */
int sw_host_alloc(void** ptr, int64_t bytes);
int sw_host_free(void* ptr);

int sw_stream_create(void** stream);
int sw_stream_destroy(void* stream);
int sw_stream_synchronize(void* stream);

/* SMs of the current device (the persistent contraction's CTA budget). */
int sw_device_sm_count(int* count);

/* Events order the streams of a sharded contraction (a chunk's collective
 * after its contraction, a partial buffer's reuse after its collective) and
 * time work on the device.  `timing` = 0 creates a lighter event that cannot
 * be timed.  sw_event_elapsed_ms waits for `end`.  No reference counterpart:
 * the reference runs one host thread on one carrier. */
int sw_event_create(void** event, int timing);
int sw_event_destroy(void* event);
int sw_event_record(void* event, void* stream);
int sw_stream_wait_event(void* stream, void* event);
int sw_event_elapsed_ms(void* start, void* end, float* ms);

/* CUDA graphs of a stream's work, for a step that repeats with the same
 * buffers (an MLP training step): capture starts on a stream from
 * sw_stream_create and ends in an executable graph; the graph can then be
 * launched on any stream, the legacy default stream (NULL) included, where it
 * is ordered with every other carrier operation.  Between begin and end the
 * calling thread may only enqueue work on that stream.  No reference
 * counterpart: the reference executes eagerly on the host. */
int sw_graph_capture_begin(void* stream);
int sw_graph_capture_end(void* stream, void** graph_exec);
int sw_graph_launch(void* graph_exec, void* stream);
int sw_graph_destroy(void* graph_exec);

/* Reads and clears the device-side error word that bounded waits and device
 * bound checks write (SW_OK if none fired).  Synchronises the device. */
int sw_device_status(int* status);

/* Exercises the device-side failure path without a fault: one thread waits,
 * with the contraction pipeline's bounded wait and a limit of limit_ns
 * (at most 1 s), on an mbarrier that nothing arrives on; the wait gives up,
 * sw_device_status then reports SW_ERR_TIMEOUT and the context stays usable.
 * No reference counterpart (the reference has no device waits). */
int sw_probe_bounded_wait(int64_t limit_ns, void* stream);

/* ---- collectives of a sharded contraction ------------------------------- */

/* NCCL behind the C ABI, for hosts that shard a contraction without
 * torch.distributed (the survey's sw_nccl_* wrappers).  Rank 0 creates the
 * id; the host hands the same SW_NCCL_ID_BYTES to every rank, and each rank,
 * with its device current, creates its communicator.  Float32 sums only: the
 * K-split reduce-scatter and an all-gather of C row blocks.  NCCL is loaded
 * at first use; without it every call returns SW_ERR_UNSUPPORTED.
 * Replaces nothing in the reference, which has no multi-device path. */
#define SW_NCCL_ID_BYTES 128
int sw_nccl_get_unique_id(uint8_t* id);
int sw_nccl_comm_init(void** comm, int world, int rank, const uint8_t* id);
/* recv[i] = sum over ranks of send[rank * recv_count + i] (recv_count per rank). */
int sw_nccl_reduce_scatter_f32(const float* send, float* recv, int64_t recv_count, void* comm, void* stream);
/* recv[r * send_count + i] = send of rank r, element i. */
int sw_nccl_all_gather_f32(const float* send, float* recv, int64_t send_count, void* comm, void* stream);
int sw_nccl_comm_destroy(void* comm);

/* The K-split over NVLink peer memory, without a collective library: every
 * rank owns a landing buffer of `world` Float32 slots (one per writer) plus
 * step flags; each rank's contraction writes its partial of every row block
 * straight into the owner's slot (sw_mx_gemm_routed: plain peer stores, no
 * TMA, no multicast), signals the owners, and each owner sums its slots in
 * rank order (the same result bit for bit on every run).  No reference
 * counterpart: the reference has no multi-device path.
 *
 * sw_ipc_alloc allocates device memory another process of the node can map
 * and writes its SW_IPC_HANDLE_BYTES-byte handle; sw_ipc_open maps a peer's
 * buffer from its handle (once per process and buffer), sw_ipc_close unmaps
 * it, sw_ipc_free releases the owner's allocation. */
#define SW_IPC_HANDLE_BYTES 64
int sw_ipc_alloc(void** ptr, int64_t bytes, uint8_t* handle);
int sw_ipc_open(const uint8_t* handle, void** ptr);
int sw_ipc_close(void* ptr);
int sw_ipc_free(void* ptr);

/* Waits on `stream` until each of the `count` 32-bit step flags at `flags`
 * (this GPU's memory, written by other ranks) reaches `target` (modulo 2^32).
 * The wait is bounded by limit_ns: past it the kernel records SW_ERR_TIMEOUT
 * for sw_device_status and returns, so a rank that died shows as a status. */
int sw_peer_wait(const uint32_t* flags, int count, uint32_t target, int64_t limit_ns, void* stream);

/* After a system-scope fence (every store the stream issued before it, peer
 * stores included, is performed first), writes `value` to each of the
 * `count` (at most 8) flags, each in some peer's memory. */
int sw_peer_signal(uint32_t* const* flags, int count, uint32_t value, void* stream);

/* out[i] = slots[i] + slots[slot_elems + i] + ... over `count` slots, in slot
 * order (Float32 adds; slot_elems a multiple of 4, 16-byte aligned). */
int sw_sum_slots_f32(const float* slots, int64_t slot_elems, int count, float* out, void* stream);

/* sw_mx_gemm_ex with Float32 results routed by row block: C rows
 * [q rows_per_dest, (q + 1) rows_per_dest) are written row-major with pitch
 * ldc starting at dest[q] (q < ndest <= 8; rows_per_dest whole 128-row tiles,
 * ndest * rows_per_dest = M; N and ldc multiples of 4).  A dest[q] may be
 * another GPU's memory mapped with sw_ipc_open: each 128 x 32 chunk of a
 * finished tile is staged in shared memory and leaves as whole 128-byte row
 * segments by plain NVLink peer stores (N under 256 stores from registers),
 * and the kernel fences them at system scope before it ends.  The walk over
 * the tiles starts with row block `first` (0 <= first < ndest) and wraps
 * around: ranks that start at different owners (rank r at r + 1, its own
 * block last) keep every GPU receiving from one writer at a time.  This is
 * the contraction half of the peer-memory K-split. */
int sw_mx_gemm_routed(int fmt, const uint8_t* a, int64_t lda, const uint8_t* scales_a,
                      const uint8_t* b, int64_t ldb, const uint8_t* scales_b,
                      float* const* dest, int ndest, int64_t rows_per_dest, int64_t ldc, int first,
                      int64_t M, int64_t N, int64_t K, int max_ctas, void* stream);

/* ---- layout-aware reductions -------------------------------------------- */

#define SW_REDUCE_SUM 0
#define SW_REDUCE_MAX 1
#define SW_REDUCE_ARGMAX 2
/* reduce_sum with accumulator_dtype=Float64: the Float32 elements are summed
 * in binary64 and the sum is rounded once to binary32
 * (src/strideweave/carriers/cpu/native/_cpu_accumulation.hpp:38-41). */
#define SW_REDUCE_SUM_F64 3

/* A two-mode (kept, reduced) Float32 view lowered to flat leaf arrays.
 * Leaves are listed first-leaf-fastest (StrideWeave's colexicographic order,
 * the order of LayoutCache::leaf_shapes, core/native/_layout_index.hpp:116-120).
 * Element (i, j) lives at carrier flat index
 *     f = offset + sum_l kept_stride[l]*i_l + sum_l reduced_stride[l]*j_l
 * and, when the carrier stores its flat space through a swizzle, at physical
 * index swizzle(f), each stage applied in order as in
 * src/strideweave/core/swizzle.py:107-117. */
typedef struct sw_reduce_plan {
    int32_t kind;          /* SW_REDUCE_* */
    int32_t kept_rank;     /* 0..SW_MAX_LEAVES (0 = a single kept element) */
    int32_t reduced_rank;  /* 1..SW_MAX_LEAVES */
    int32_t swizzle_rank;  /* 0..SW_MAX_SWIZZLE */
    int64_t offset;
    int64_t kept_shape[SW_MAX_LEAVES];
    int64_t kept_stride[SW_MAX_LEAVES];
    int64_t reduced_shape[SW_MAX_LEAVES];
    int64_t reduced_stride[SW_MAX_LEAVES];
    int32_t swizzle_bits[SW_MAX_SWIZZLE];
    int32_t swizzle_base[SW_MAX_SWIZZLE];
    int32_t swizzle_shift[SW_MAX_SWIZZLE];
} sw_reduce_plan;

/* out[i] for every kept ordinal i (canonical 1-mode result, stride 1):
 * SUM -> float, MAX -> float (bit-exact with cpu.reduce_max), ARGMAX -> int32
 * (bit-exact with cpu.argmax).  `x_size` is the carrier size in elements and
 * bounds every address.
 * Replaces CpuReduceSumOperation::_forward
 * (src/strideweave/carriers/cpu/native/ops/reduce_sum.cpp:30-118) and
 * CpuFloatReductionOperation<Kind>::_forward for reduce_max / argmax
 * (src/strideweave/carriers/cpu/native/_cpu_reduction.hpp:47-120). */
int sw_reduce_f32(const sw_reduce_plan* plan, const float* x, int64_t x_size,
                  void* out, void* stream);

/* sw_reduce_f32 without any device allocation.  This entry point has no
 * counterpart in the reference: it exists for callers that cannot let a
 * library allocate device memory, such as an engine that has already divided
 * the whole device among its own pools, or a process whose memory budget is
 * fixed and audited per allocation.  Same plans, results and errors as
 * sw_reduce_f32, except that the scratch of a split column reduction lives in
 * a 2 MiB array compiled into the library, which every GPU that loads the
 * library keeps until the process exits; a reduction needing more scratch
 * (only possible on devices with more than 255 SMs) fails with
 * SW_ERR_UNSUPPORTED.  The first call on each device looks up the array's
 * device address, so make that first call before any stream capture.  All
 * calls share the one array and each clears its counters on its own stream:
 * calls that overlap on the GPU (other streams, other host threads) race and
 * produce wrong results, so order them on one stream.  The array's address
 * is looked up once per device and kept for the life of the process: after a
 * cudaDeviceReset (or any reset of the primary context) this entry point is
 * not supported. */
int sw_reduce_f32_noalloc(const sw_reduce_plan* plan, const float* x, int64_t x_size,
                          void* out, void* stream);

/* Gradient of sw_reduce_f32 with respect to its input (the VJP of
 * CpuReduceSumOperation::backward, ops/reduce_sum.cpp:120-150, and of
 * CpuFloatReductionOperation<Kind>::backward for reduce_max,
 * _cpu_reduction.hpp:135-196):
 *   SUM: grad_in[i, j] = grad_out[i] for every j;
 *   MAX: grad_in[i, j] = grad_out[i] / w_i where x[i, j] equals the row's
 *        maximum (w_i = how many do), 0 elsewhere; every element of a row
 *        whose maximum is NaN gets NaN.
 * `plan` describes the forward input view x (`x` may be NULL for SUM);
 * `grad_plan` has the same leaf extents and places grad_in (kind ignored).
 * grad_out holds one float per kept ordinal (the canonical result layout). */
int sw_reduce_backward_f32(const sw_reduce_plan* plan, const float* x,
                           int64_t x_size, const float* grad_out,
                           float* grad_in, const sw_reduce_plan* grad_plan,
                           int64_t grad_size, void* stream);

/* Copies a two-mode Float32 view into another two-mode placement:
 * dst[dst.offset + kept_d(i) + reduced_d(j)] = src at (i, j) of `src_plan`
 * (each flat index through its own plan's swizzle), for every (i, j).  Both
 * plans' leaves must have the same mode sizes; `kind` fields are ignored.
 * Any 32-bit element copies bit for bit (Int32 views too).  This is how the carrier
 * materialises views no kernel walks directly (the reference's
 * _physical_values_for_layout / _detached_tensor_like,
 * src/strideweave/carriers/operation_helpers.py:194-245), and how it scatters
 * a tensor onto another through a mapping layout in one launch
 * (CpuCarrier::scatter, src/strideweave/carriers/cpu/native/
 * _cpu_carrier.hpp:521-540). */
int sw_copy_view_f32(const sw_reduce_plan* src_plan, const float* src,
                     int64_t src_size, const sw_reduce_plan* dst_plan,
                     float* dst, int64_t dst_size, void* stream);

/* ---- elementwise work around the contractions (the MLP step) ------------- */

#define SW_EW_GELU 0      /* out = a * Phi(a), the erf GELU                    */
#define SW_EW_GELU_GRAD 1 /* out = b * d/da (a * Phi(a)); b = upstream grad    */
#define SW_EW_AXPY 2      /* out = a + alpha * b (out may alias a: SGD update) */

/* Elementwise Float32 map over n contiguous elements.  GELU follows the
 * reference's erf form, gelu(x) = x / 2 * (1 + erf(x / sqrt 2))
 * (src/strideweave/carriers/cpu/native/_cpu_operation.hpp:33-40); AXPY is the
 * SGD update the reference applies element by element
 * (src/strideweave/nn/optim.py:45-80). */
int sw_elementwise_f32(int op, int64_t n, const float* a, const float* b,
                       float* out, float alpha, void* stream);

/* Mean squared error of n contiguous pairs: loss[0] = sum((p - t)^2) / n
 * (float accumulation; MSELoss, src/strideweave/nn/modules.py:129-200).
 * With grad != NULL also grad[i] = u * 2 * (p[i] - t[i]) / n, where u is
 * upstream[0] (the loss gradient on the device) or 1 when upstream is NULL. */
int sw_mse_f32(int64_t n, const float* pred, const float* target, float* loss,
               const float* upstream, float* grad, void* stream);

/* ---- MX (OCP Microscaling v1.0) quantise / dequantise ------------------- */

#define SW_MX_E4M3 1 /* MXFP8_E4M3: 1 byte per element              */
#define SW_MX_E2M1 2 /* MXFP4: 2 elements per byte, even k in the low nibble */

/* Scale-plane placements (E8M0 bytes, one per 32-element block along K). */
#define SW_SCALES_ROWMAJOR 0 /* scales[r * ld_scales + kb]                 */
#define SW_SCALES_TC128 1    /* 128-row x 4-block atoms, see sw_mx_scale_index */

/* Byte offset of scale (row r, block kb) in the SW_SCALES_TC128 placement of a
 * plane with `kblocks` 32-blocks per row: atoms of 128 rows x 4 blocks (512 B)
 * ordered K-block-fastest within a 128-row group, inside an atom
 * (r % 32) * 16 + ((r / 32) % 4) * 4 + kb % 4.  This is the StrideWeave layout
 * ((32,4,R/128),(4,KB/4)) : ((16,4,512*ceil(KB/4)),(1,512)), and the order
 * tcgen05.cp .32x128b.warpx4 consumes. Padding blocks hold 127 (1.0). */
int64_t sw_mx_scale_index(int64_t r, int64_t kb, int64_t kblocks);
/* Bytes of a SW_SCALES_TC128 scale plane for rows x kblocks (padded). */
int64_t sw_mx_scale_bytes_tc128(int64_t rows, int64_t kblocks);

/* Quantise X[rows, cols] (element (r, c) at x[r*ld_x_row + c*ld_x_col],
 * Float32) into MX blocks of 32 along `cols`.  Payload row r starts at byte
 * r*ld_payload (E2M1: byte c/2 of the row holds element c, even c low nibble).
 * Bit-exact with the OCP MX v1.0 restatement in oracle/sw_oracle.c.
 * There is no reference counterpart: the reference declares MXFP8_E4M3 and
 * MXFP4 as descriptors only (src/strideweave/carriers/_dtype/builtins.py:39-52). */
int sw_mx_quantize(int fmt, const float* x, int64_t rows, int64_t cols,
                   int64_t ld_x_row, int64_t ld_x_col, uint8_t* payload,
                   int64_t ld_payload, uint8_t* scales, int scale_layout,
                   int64_t ld_scales, void* stream);

/* sw_mx_quantize over any hierarchical two-mode Float32 view: `view` is the
 * lowered layout (its kept leaves give the rows, its reduced leaves the
 * quantised axis, `kind` ignored), carrier flat index f holding element
 * (r, c) as in sw_reduce_plan, through the carrier swizzle, within a carrier
 * of x_size elements (checked before any launch).  Same planes, bit for bit,
 * as sw_mx_quantize on the same logical values.  This is how a tiled or
 * swizzled Float32 tensor (src/strideweave/core/layout.py:1374-1546,
 * src/strideweave/core/swizzle.py:107-117) is quantised where it lies. */
int sw_mx_quantize_view(int fmt, const sw_reduce_plan* view, const float* x,
                        int64_t x_size, uint8_t* payload, int64_t ld_payload,
                        uint8_t* scales, int scale_layout, int64_t ld_scales,
                        void* stream);

/* Rewrites a row-major scale plane (scales[r * ld_src + kb], rows x kblocks)
 * into the SW_SCALES_TC128 placement sw_mx_gemm reads, padding with 127.
 * An MX tensor whose rows or blocks are not whole 128 x 4 atoms keeps its
 * scales row-major (the reference's LevelExtent(0, 32) rule wants the scale
 * plane's shape to be exactly rows x K/32); its contraction goes through this. */
int sw_mx_scales_to_tc128(const uint8_t* src, int64_t ld_src, int64_t rows,
                          int64_t kblocks, uint8_t* dst, void* stream);

/* What sw_mx_quantize_dual quantises: S = x, gelu(x), or x * gelu'(h). */
#define SW_XF_NONE 0
#define SW_XF_GELU 1      /* S = x * Phi(x), as SW_EW_GELU                         */
#define SW_XF_GELU_GRAD 2 /* S = x * d/dh (h * Phi(h)), as SW_EW_GELU_GRAD (a = h) */

/* Quantises S[rows, cols] (S[i, j] from x[i*ld_x + j], and h likewise) both
 * ways in one pass: the "row planes" hold S blocked along cols (the operand
 * [rows, cols]), the "column planes" S blocked along rows (the operand
 * [cols, rows], i.e. S transposed).  Either plane pair may be NULL.  The
 * planes are bit-identical to sw_elementwise_f32 followed by two
 * sw_mx_quantize calls; this is what one activation of an MLP layer needs for
 * its forward and its weight-gradient contraction.  Requires rows % 32 == 0,
 * cols % 128 == 0, ld_x % 4 == 0 and 16-byte aligned x and h, else
 * SW_ERR_UNSUPPORTED (use the separate calls).  No reference counterpart
 * beyond sw_mx_quantize's: it fuses the GELU of
 * src/strideweave/carriers/cpu/native/_cpu_operation.hpp:33-40 into it. */
int sw_mx_quantize_dual(int fmt, int transform, const float* x, const float* h,
                        int64_t rows, int64_t cols, int64_t ld_x,
                        uint8_t* payload_r, int64_t ld_payload_r, uint8_t* scales_r,
                        int scale_layout_r, int64_t ld_scales_r,
                        uint8_t* payload_c, int64_t ld_payload_c, uint8_t* scales_c,
                        int scale_layout_c, int64_t ld_scales_c, void* stream);

/* Exact inverse image: out[r*ld_out + c] = element * 2^(scale-127)
 * (NaN where the scale byte is 0xFF). */
int sw_mx_dequantize(int fmt, const uint8_t* payload, int64_t ld_payload,
                     const uint8_t* scales, int scale_layout, int64_t ld_scales,
                     int64_t rows, int64_t cols, float* out, int64_t ld_out,
                     void* stream);

/* ---- block-scaled contraction ------------------------------------------ */

#define SW_OUT_F32 0
#define SW_OUT_BF16 1

/* C[m, n] = sum_k A[m, k] * B[n, k] over MX operands, fp32 accumulation.
 * A: payload rows of K elements (K-major) with row pitch lda bytes, scales in
 * the SW_SCALES_TC128 placement for M x K/32 (whole atoms: its padding blocks
 * must hold finite scales, as sw_mx_quantize writes them); B likewise for
 * N x K/32.  C[m, n] is written at c[m*ldc_m + n*ldc_n] (elements of
 * out_dtype); either pitch may be 1 (row- or column-major).  When `beta_one`
 * is non-zero the result is added to C's current fp32 contents instead of
 * replacing them.  Any M and N (a ragged last tile is clipped); K a positive
 * multiple of 32 (whole MX blocks).  Requires fmt_a == fmt_b and 16-byte
 * aligned payload pointers and pitches.
 * Replaces CpuMatmulOperation::_forward
 * (src/strideweave/carriers/cpu/native/ops/matmul.cpp:45-113) for MX operands,
 * which the reference refuses (operation_policy.py:1407-1440). */
int sw_mx_gemm(int fmt_a, int fmt_b, const uint8_t* a, int64_t lda,
               const uint8_t* scales_a, const uint8_t* b, int64_t ldb,
               const uint8_t* scales_b, void* c, int out_dtype, int64_t ldc_m,
               int64_t ldc_n, int64_t M, int64_t N, int64_t K, int beta_one,
               void* stream);

/* sw_mx_gemm on at most max_ctas SMs (0 = every SM).  The persistent kernel
 * otherwise holds one CTA with ~220 KB of shared memory on every SM, so a
 * kernel launched beside it on another stream (an NCCL collective) cannot
 * start until it ends; leaving a few SMs free lets a K-split's
 * reduce-scatter overlap the next chunk's contraction. */
int sw_mx_gemm_ex(int fmt_a, int fmt_b, const uint8_t* a, int64_t lda,
                  const uint8_t* scales_a, const uint8_t* b, int64_t ldb,
                  const uint8_t* scales_b, void* c, int out_dtype, int64_t ldc_m,
                  int64_t ldc_n, int64_t M, int64_t N, int64_t K, int beta_one,
                  int max_ctas, void* stream);

/* `batch` independent contractions C_p = A_p B_p^T (p < batch) in one
 * persistent launch: the batched block-scaled GEMM that a batched einsum over
 * MX operands lowers to, in place of the union product the reference
 * materialises (einops/__init__.py:459-475).  The operands are stacks:
 * A_p is rows [p M, (p + 1) M) of one [batch M, K] MX operand (payload pitch
 * lda, SW_SCALES_TC128 scales of the whole stack), B_p rows [p N, (p + 1) N)
 * of one [batch N, K] operand.  C_p starts batch_stride_c elements after
 * C_(p-1) and has the pitches ldc_m / ldc_n.  The C_p must be disjoint:
 * with batch > 1, the three strides (batch_stride_c, ldc_m, ldc_n), taken in
 * increasing order, must each exceed the span of the modes below them
 * (stacked blocks and interleaved problems both qualify); other placements
 * are refused with SW_ERR_INVALID.  Row-major
 * results with batch_stride_c = M ldc_m and column-major ones with
 * batch_stride_c = N ldc_n are written by the staged epilogues; any other
 * stride stores from registers.  M and N must be multiples of 128 (whole
 * scale atoms per problem).  Other arguments and errors as sw_mx_gemm. */
int sw_mx_gemm_batched(int fmt_a, int fmt_b, const uint8_t* a, int64_t lda,
                       const uint8_t* scales_a, const uint8_t* b, int64_t ldb,
                       const uint8_t* scales_b, void* c, int out_dtype,
                       int64_t ldc_m, int64_t ldc_n, int64_t batch_stride_c,
                       int64_t batch, int64_t M, int64_t N, int64_t K,
                       int beta_one, void* stream);

/* ---- Float32 contraction (the reference's own plan) ---------------------- */

/* C[m, n] = sum_k A[m, k] * B[n, k], Float32 products accumulated in Float32,
 * for arbitrary element strides (a[m*sam + k*sak], b[n*sbn + k*sbk],
 * c[m*scm + n*scn]).
 * Replaces CpuMatmulOperation::_forward
 * (src/strideweave/carriers/cpu/native/ops/matmul.cpp:45-113) for the
 * BINARY32 / FLOATING / Float32 plan (operation_policy.py:784-815). */
int sw_matmul_f32(const float* a, int64_t sam, int64_t sak, const float* b,
                  int64_t sbn, int64_t sbk, float* c, int64_t scm, int64_t scn,
                  int64_t M, int64_t N, int64_t K, void* stream);

/* A batch of sw_matmul_f32 contractions in one launch: contraction z reads
 * a + z*sab, b + z*sbb and writes c + z*scb.  Serves batched einsum without
 * the union product the reference materialises for batch symbols
 * (src/strideweave/einops/__init__.py:459-475: align over the union index
 * space, elementwise_mul, reduce_sum). */
int sw_matmul_f32_batched(const float* a, int64_t sab, int64_t sam, int64_t sak,
                          const float* b, int64_t sbb, int64_t sbn, int64_t sbk,
                          float* c, int64_t scb, int64_t scm, int64_t scn,
                          int64_t batch, int64_t M, int64_t N, int64_t K,
                          void* stream);

#define SW_ACC_F32 0 /* the default FLOATING / Float32 accumulator              */
#define SW_ACC_F64 1 /* accumulator_dtype=Float64: binary32 products summed in
                      * binary64, rounded once (operation_policy.py:784-815) */

/* sw_matmul_f32_batched with a chosen accumulator (SW_ACC_*): the widened
 * plan of CpuMatmulOperation (_cpu_accumulation.hpp:38-41), forward and
 * backward alike. */
int sw_matmul_f32_batched_ex(const float* a, int64_t sab, int64_t sam, int64_t sak,
                             const float* b, int64_t sbb, int64_t sbn, int64_t sbk,
                             float* c, int64_t scb, int64_t scm, int64_t scn,
                             int64_t batch, int64_t M, int64_t N, int64_t K,
                             int accumulator, void* stream);

/* ---- binary elementwise -------------------------------------------------- */

#define SW_BIN_MUL 0

/* out[o(i)] = a[a(i)] * b[b(i)] for every logical index i of `rank` leaves
 * (first leaf fastest, at most 16) shared by the three views, each with its
 * own strides (0 on a broadcast leaf) and offset; every address is checked
 * against its carrier's size first.  Replaces the forward of the reference's
 * elementwise_mul, CpuElementwiseMulOperation::_forward
 * (src/strideweave/carriers/cpu/native/ops/elementwise_mul.cpp:10-16 via
 * _cpu_binary.hpp:85-130), products rounded to binary32. */
int sw_binary_f32(int op, int rank, const int64_t* shape,
                  const float* a, int64_t a_offset, const int64_t* a_stride, int64_t a_size,
                  const float* b, int64_t b_offset, const int64_t* b_stride, int64_t b_size,
                  float* out, int64_t out_offset, const int64_t* out_stride, int64_t out_size,
                  void* stream);

/* The elementwise arithmetic the reference's nn modules compose (a Linear's
 * bias add, an MSE loss's difference, square and mean scale, and their
 * gradients), each a binary32 operation per element as the CPU carrier's
 * kernels do it. */
#define SW_MAP_ADD 0      /* a + b: CpuAddOperation (ops/add.cpp)                          */
#define SW_MAP_SUB 1      /* a - b: CpuSubOperation (ops/sub.cpp)                          */
#define SW_MAP_MUL 2      /* a * b: the tensor-tensor mul (ops/scalar_mul.cpp)             */
#define SW_MAP_SCALE 3    /* a * scalar: CpuScalarMulOperation (ops/scalar_mul.cpp)        */
#define SW_MAP_POW 4      /* pow(a, scalar): the tensor ** weak-scalar CpuPowOperation     */
#define SW_MAP_POW_GRAD 5 /* a * scalar * pow(b, scalar - 1): that pow's gradient (ops/pow.cpp:160-175),
                           * a = incoming gradient, b = base                               */

/* sw_binary_f32 generalised to the SW_MAP_* operations: the same shared-leaf
 * walk and bounds checks; SCALE and POW read only `a` (b and its strides may
 * be NULL).  pow with exponent 2 or 1 is the exact product the reference's
 * std::pow gives; other exponents use the device powf. */
int sw_map_f32(int op, int rank, const int64_t* shape,
               const float* a, int64_t a_offset, const int64_t* a_stride, int64_t a_size,
               const float* b, int64_t b_offset, const int64_t* b_stride, int64_t b_size,
               float* out, int64_t out_offset, const int64_t* out_stride, int64_t out_size,
               float scalar, void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* STRIDEWEAVE_B200_H */
