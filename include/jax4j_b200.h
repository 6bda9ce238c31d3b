/*
 * jax4j_b200 -- C ABI of the B200 (sm_100a) engine behind JAX4J's engine SPI.
 *
 * One entry point per reference SPI operation. A thin binding (Java FFM in the JAX4J tree, or
 * ctypes here) maps each ComputeBackend / QuantizedOps method to one call below, as the
 * reference's CudaRuntime maps its methods onto cu* driver calls. Reference interfaces are cited
 * by their path inside the jax4j project, with these prefixes:
 *   core/ = jax4j-core/src/main/java/com/nablatensor/jax4j/
 *   cuda/ = jax4j-engine-cuda/src/main/java/com/nablatensor/jax4j/
 *
 * Conventions
 *   - Every function returns an int status (J4B_OK == 0). On failure j4b_last_error() returns a
 *     message for the calling thread. J4B_EINVAL is raised for shape/argument violations before
 *     any launch (the reference's IllegalArgumentException), J4B_EUNSUPPORTED for unsupported
 *     types (UnsupportedOperationException), J4B_ECUDA for driver/runtime failures
 *     (RuntimeException "<op> failed: <CUDA error>").
 *   - Device buffers are plain device addresses carried as uint64_t (j4b_buf). Any allocator may
 *     produce them (j4b_alloc, or a framework such as PyTorch); f32 tensors are dense row-major.
 *   - Launches are asynchronous on the given stream (a cudaStream_t passed as void*). A NULL
 *     stream selects the engine's own per-device non-blocking stream created by j4b_init; pass
 *     cudaStreamLegacy ((void*)1) to mean the legacy default stream.
 *   - Shapes are (const int64_t* dims, int rank); rank <= 8.
 */
#ifndef JAX4J_B200_H
#define JAX4J_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define J4B_OK 0
#define J4B_EINVAL 1
#define J4B_ENOMEM 2
#define J4B_ECUDA 3
#define J4B_EUNSUPPORTED 4
#define J4B_ENOTINIT 5
#define J4B_ETIMEOUT 6

typedef uint64_t j4b_buf;          /* device address of a dense f32 buffer */
typedef void* j4b_stream;          /* cudaStream_t; NULL = engine stream of the device */
typedef struct j4b_qweight* j4b_qweight_t; /* opaque quantized matrix (QuantizedOps buffer) */

/* GGUF type ids: core/tensor/QuantType.java:4-13 */
#define J4B_Q4_0 2
#define J4B_Q8_0 8
#define J4B_Q4_K 12
#define J4B_Q6_K 14
#define J4B_Q2_0 42

/* Op codes: the ordinal order of core/tensor/Op.java:19-23 (the reference's CUDA kernels
 * switch on the same enum, cuda/backend/cuda/CudaBackend.java:1053-1079). */
#define J4B_ADD 0
#define J4B_SUB 1
#define J4B_MUL 2
#define J4B_DIV 3
#define J4B_MAX 4
#define J4B_MIN 5
#define J4B_NEG 6
#define J4B_EXP 7
#define J4B_LOG 8
#define J4B_SQRT 9
#define J4B_RSQRT 10
#define J4B_TANH 11
#define J4B_SIGMOID 12
#define J4B_RELU 13
#define J4B_ABS 14
#define J4B_SIGN 15

/* Engine counters; the names follow the reference GPU backends' diagnostics() records
 * (core/tensor/spi/GpuTensorBackend.java, read by core/tensor/bench/GpuComparison.java:35-56). */
typedef struct j4b_diagnostics {
  uint64_t dispatches;    /* kernel launches issued by the engine */
  uint64_t allocations;   /* device allocations made by the engine */
  uint64_t releases;      /* device frees made by the engine */
  uint64_t h2d_bytes;     /* host->device bytes copied by j4b_h2d / uploads */
  uint64_t d2h_bytes;     /* device->host bytes copied by j4b_d2h */
  uint64_t compilations;  /* runtime kernel compilations (fused tapes) */
} j4b_diagnostics;

/* ---- lifecycle: cuda/backend/cuda/CudaRuntime.java:140-211 (cuInit, context on device 0) --- */

/* Initialises the listed devices (NULL/0 = device 0). Idempotent. */
int j4b_init(const int* devices, int n);
/* ComputeBackend.isAvailable (core/tensor/spi/ComputeBackend.java:43): never fails; count 0
 * when no usable GPU exists. */
int j4b_device_count(int* count);
int j4b_device_name(int dev, char* buf, size_t len);
int j4b_sm_count(int dev, int* count);
int j4b_get_stream(int dev, j4b_stream* stream);
/* ComputeBackend.sync (core/tensor/spi/ComputeBackend.java:276-277) */
int j4b_sync(int dev);
int j4b_last_error(char* buf, size_t len);
int j4b_get_diagnostics(j4b_diagnostics* out);

/* ---- memory: CudaRuntime.java:252-290 (malloc/pool), :432-485 (HtoD/DtoH) ---- */

int j4b_alloc(int dev, size_t bytes, j4b_buf* out);
/* Stream-ordered free on the device's engine stream: safe to call from any thread, and on a
 * value of 0 (no-op). Replaces the reference's pending-free queue (CudaRuntime.java:407-430). */
int j4b_free(j4b_buf buf);
/* ComputeBackend.upload (ComputeBackend.java:48) */
int j4b_h2d(j4b_buf dst, const void* src, size_t bytes, j4b_stream stream);
/* ComputeBackend.download (ComputeBackend.java:87): synchronises the stream first. */
int j4b_d2h(void* dst, j4b_buf src, size_t bytes, j4b_stream stream);
int j4b_d2d(j4b_buf dst, j4b_buf src, size_t bytes, j4b_stream stream);

/* ---- dense SPI primitives (core/tensor/spi/ComputeBackend.java:48-280) ---- */

/* full: ComputeBackend.java:78-85 */
int j4b_fill(j4b_buf out, int64_t n, float value, j4b_stream s);
/* binary: ComputeBackend.java:89 (equal element counts; CpuBackend.java:61-94 semantics) */
int j4b_binary(int op, j4b_buf a, j4b_buf b, j4b_buf out, int64_t n, j4b_stream s);
/* scalar: ComputeBackend.java:91 (value cast to float first, CpuBackend.java:101) */
int j4b_scalar(int op, j4b_buf a, double value, j4b_buf out, int64_t n, j4b_stream s);
/* unary: ComputeBackend.java:93 */
int j4b_unary(int op, j4b_buf a, j4b_buf out, int64_t n, j4b_stream s);
/* transpose: ComputeBackend.java:95 (rank 2) */
int j4b_transpose(j4b_buf a, j4b_buf out, int64_t rows, int64_t cols, j4b_stream s);
/* reduceSum / reduceMax: ComputeBackend.java:150-153 (out is one float) */
int j4b_reduce_sum(j4b_buf a, int64_t n, j4b_buf out, j4b_stream s);
int j4b_reduce_max(j4b_buf a, int64_t n, j4b_buf out, j4b_stream s);
/* sumAxis / maxAxis / argMaxAxis: ComputeBackend.java:158-172, the tensor viewed as
 * [outer, axis, inner]; out is [outer, inner] (keepDims only changes the shape). sumAxis0
 * (ComputeBackend.java:156) is outer = 1. */
int j4b_sum_axis(j4b_buf a, int64_t outer, int64_t axis, int64_t inner, j4b_buf out,
                 j4b_stream s);
int j4b_max_axis(j4b_buf a, int64_t outer, int64_t axis, int64_t inner, j4b_buf out,
                 j4b_stream s);
int j4b_argmax_axis(j4b_buf a, int64_t outer, int64_t axis, int64_t inner, j4b_buf out,
                    j4b_stream s);
/* maxAxisBackward: ComputeBackend.java:174-177 */
int j4b_max_axis_backward(j4b_buf upstream, j4b_buf input, int64_t outer, int64_t axis,
                          int64_t inner, j4b_buf out, j4b_stream s);
/* broadcastTo: ComputeBackend.java:205-206 (numpy rules, any rank <= 8) */
int j4b_broadcast_to(j4b_buf a, const int64_t* src_dims, int src_rank, const int64_t* dst_dims,
                     int dst_rank, j4b_buf out, j4b_stream s);
/* reindex / scatterAdd: ComputeBackend.java:247-274. map is a device int32 array; -1 means
 * zero (reindex) or discard (scatterAdd). The kernels treat entries outside [-1, n) as -1; the
 * binding validates the static map once, on the host, when it uploads it (the reference's
 * "index out of bounds" check, ComputeBackend.java:254-255, 269-270). */
int j4b_reindex(j4b_buf a, int64_t n_src, j4b_buf map, int64_t n_dst, j4b_buf out,
                j4b_stream s);
int j4b_scatter_add(j4b_buf a, int64_t n_src, j4b_buf map, int64_t n_dst, j4b_buf out,
                    j4b_stream s);
/* Full sum that allocates nothing (no counterpart in the reference). For callers that cannot
 * allocate device memory while they run -- a host that fixes its device-memory budget up front
 * (a JVM handing the engine a pre-sized arena), a serving loop that must not take the
 * allocator's locks or fail for lack of memory mid-request -- where j4b_reduce_sum would
 * allocate its block partials. The input must be on the output's device (J4B_EINVAL otherwise). Same result as j4b_reduce_sum (double accumulation, one float
 * out) within the sums' rounding. Its scratch is a static device array of 512 KiB per GPU that
 * loads the library, held until exit, so n is limited to 134,217,728 elements (J4B_EINVAL
 * above that). The first call on a device looks the array up and zeroes its counter, so make
 * it before any stream capture. All calls share the array: calls that overlap on the GPU race. */
int j4b_reduce_sum_noalloc(j4b_buf a, int64_t n, j4b_buf out, j4b_stream s);
/* reluBackward: ComputeBackend.java:202-203 */
int j4b_relu_backward(j4b_buf upstream, j4b_buf input, j4b_buf out, int64_t n, j4b_stream s);
/* randomUniform / randomNormal: ComputeBackend.java:50-76 (bit-exact uniforms) */
int j4b_random_uniform(int64_t seed, int64_t counter, j4b_buf out, int64_t n, j4b_stream s);
int j4b_random_normal(int64_t seed, int64_t counter, j4b_buf out, int64_t n, j4b_stream s);
/* matmul / batchedMatmul: ComputeBackend.java:97-101. out[b] = a[b] (m x k) . b[b] (k x n),
 * row-major f32. precision 0 = fp32-accurate (rel 1e-4): SIMT for small shapes, the tcgen05
 * tensor cores with a 3-term bf16 split (hi.hi + hi.lo + lo.hi) when m n k >= 2^24;
 * 1 = bf16 operands on the tensor cores (rel 1e-2); 2 = the 3-term split on the tensor cores
 * at any size. */
int j4b_matmul(j4b_buf a, j4b_buf b, j4b_buf out, int64_t batch, int64_t m, int64_t k,
               int64_t n, int precision, j4b_stream s);

/* ---- conv2d / conv2dGradInput / conv2dGradWeight: ComputeBackend.java:191-200 (CPU semantics
 * CpuBackend.java:479-609). ConvSpec (core/tensor/ConvSpec.java) as plain ints: images NCHW
 * flattened per row, x [batch, in_c*in_h*in_w], w [out_c, in_c*kernel*kernel], output
 * [batch, out_c*out_h*out_w] with out_h = (in_h + 2 pad - kernel) / stride + 1 (likewise out_w).
 * precision as j4b_matmul (0 = fp32-accurate). Invalid specs: J4B_EINVAL with ConvSpec's
 * messages. */
int j4b_conv2d(j4b_buf x, j4b_buf w, j4b_buf out, int64_t batch, int in_c, int in_h, int in_w,
               int out_c, int kernel, int stride, int pad, int precision, j4b_stream s);
int j4b_conv2d_grad_input(j4b_buf upstream, j4b_buf w, j4b_buf out, int64_t batch, int in_c,
                          int in_h, int in_w, int out_c, int kernel, int stride, int pad,
                          int precision, j4b_stream s);
int j4b_conv2d_grad_weight(j4b_buf x, j4b_buf upstream, j4b_buf out, int64_t batch, int in_c,
                           int in_h, int in_w, int out_c, int kernel, int stride, int pad,
                           int precision, j4b_stream s);

/* ---- QuantizedOps: core/tensor/spi/QuantizedOps.java:19-34 ---- */

/* supportedQuantTypes (QuantizedOps.java:21): writes up to cap ids, returns the count in *n. */
int j4b_quant_supported(int* ids, int cap, int* n);
/* Bytes of a rows x cols matrix in GGUF blocks (QuantType.byteSizeFor, QuantType.java:46-53). */
int j4b_quant_bytes(int ggml_type, int64_t rows, int64_t cols, int64_t* bytes);
/* uploadQuantized (QuantizedOps.java:23-24): copies a host GGUF blob to the device and repacks
 * it into the engine's tensor-core fragment layout (same byte count). */
int j4b_quant_upload(int dev, const void* blocks, size_t bytes, int ggml_type, int64_t rows,
                     int64_t cols, j4b_qweight_t* out);
/* Same, from a GGUF blob already resident on the device (e.g. written by j4b_quantize). */
int j4b_quant_upload_device(int dev, j4b_buf blocks, size_t bytes, int ggml_type, int64_t rows,
                            int64_t cols, j4b_qweight_t* out);
int j4b_quant_free(j4b_qweight_t w);
int j4b_quant_shape(j4b_qweight_t w, int* ggml_type, int64_t* rows, int64_t* cols);
/* quantMatvec / quantMatvecAdd (QuantizedOps.java:26-30), batched: x [batch, cols] f32,
 * add [batch, rows] f32 or 0, y [batch, rows] f32. batch = 1 is the reference call. The
 * dequant-GEMV (fp16 fragments of the codes, x split into fp16 hi + lo, fp32 accumulation) in
 * passes of up to 16 rows of x; from 33 rows (Q8_0) or 49 rows (Q4_0, Q4_K) one pass of the fused
 * dequant-GEMM below in its fp32-accurate mode. Either way relative error ~1e-5 (bar 1e-4). */
int j4b_quant_matvec(j4b_qweight_t w, j4b_buf x, j4b_buf add, j4b_buf y, int64_t batch,
                     j4b_stream s);
/* The same with HOST buffers (QuantizedOps.java:26-30 as a host caller makes it: upload x, the
 * product, download y): x [batch, cols] and y [batch, rows] f32 in host memory, batch 1..16.
 * Everything is queued on the stream; y is valid once the stream is synchronised. Page-locked
 * buffers (cudaHostAlloc / cudaMallocHost, e.g. torch pin_memory) are used in place: a kernel
 * reads x over PCIe and the GEMV stores y into host memory; pageable buffers go through copies.
 * Device staging for x belongs to the weight (allocated by the first call), so calls on one
 * weight must not overlap. */
int j4b_quant_matvec_host(j4b_qweight_t w, const float* x, int64_t batch, float* y, j4b_stream s);
/* Prefill projection (no reference counterpart: the reference only has the rank-1 quantMatvec):
 * y [m, rows] = x [m, cols] . W^T, f32 row-major, on the tcgen05 tensor cores. precision
 * 1 = bf16 operands (rel 1e-2); 0 or 2 = 3-term bf16 split of both operands (rel 1e-4). Q8_0,
 * Q4_0, Q4_K: the weight's blocks are decoded inside the GEMM, into the tensor cores' shared-
 * memory operand tiles (no dequantised copy); Q6_K, Q2_0: decoded into stream-ordered scratch
 * first. x is converted to bf16 in stream-ordered scratch. */
int j4b_quant_gemm(j4b_qweight_t w, j4b_buf x, j4b_buf y, int64_t m, int precision, j4b_stream s);
/* quantGatherRow (QuantizedOps.java:32-33): bit-exact dequantised row, out [cols] f32. */
int j4b_quant_gather_row(j4b_qweight_t w, int64_t row, j4b_buf out, j4b_stream s);
/* Encoder (no reference counterpart; producers of GGUF data): w [rows, cols] f32 on the device
 * -> GGUF blocks on the device. Byte-identical to the published block encoders restated in the
 * oracle. */
int j4b_quantize(int ggml_type, j4b_buf w, int64_t rows, int64_t cols, j4b_buf out_blocks,
                 j4b_stream s);

/* ---- Collectives over NVLink peer memory (no reference counterpart: the reference has no
 * multi-GPU path). One process per GPU; each rank allocates one buffer, exchanges the 64-byte
 * IPC handles out of band (e.g. torch.distributed), maps the others and builds a group. A
 * `channel` (0..15) is an independent sequence of collective calls; every rank must make the
 * same calls on a channel in the same order. Waits are bounded (about a second); a wait that
 * gives up sets the group status (j4b_peer_status) instead of hanging. ---- */
typedef struct j4b_peer_group j4b_peer_group;
int j4b_peer_alloc(int dev, size_t bytes, j4b_buf* local, uint8_t* ipc_handle_64);
int j4b_peer_open(int dev, const uint8_t* ipc_handle_64, j4b_buf* remote);
int j4b_peer_close(j4b_buf remote);
int j4b_peer_free(j4b_buf local);
/* bases[r] = rank r's buffer as mapped in this process (the local one for r == rank). */
int j4b_peer_group_create(int dev, int nranks, int rank, const j4b_buf* bases, size_t bytes,
                          j4b_peer_group** out);
int j4b_peer_group_free(j4b_peer_group* g);
int j4b_peer_status(j4b_peer_group* g, int* status);
/* Row-sharded quantMatvec fused with its all-gather: this rank's W holds rows
 * [rank*rows, (rank+1)*rows) of the whole matrix; the GEMV stores its outputs straight into
 * every rank's buffer and y_all [batch, rows * nranks] receives the gathered result. batch <= 16. */
int j4b_quant_matvec_allgather(j4b_qweight_t w, j4b_buf x, j4b_buf add, j4b_buf y_all, int64_t batch,
                               j4b_peer_group* g, int channel, j4b_stream s);
/* The same with host buffers, as j4b_quant_matvec_host: x [batch, cols] and the gathered
 * y_all [batch, rows * nranks] in host memory (page-locked ones are read and written in place
 * by the kernels). */
int j4b_quant_matvec_allgather_host(j4b_qweight_t w, const float* x, int64_t batch, float* y_all,
                                    j4b_peer_group* g, int channel, j4b_stream s);
/* A host-buffer call (g = NULL: j4b_quant_matvec_host; else j4b_quant_matvec_allgather_host on
 * `channel`) recorded once as a CUDA graph; each run replays it with one launch on the stream (a
 * decode loop's per-step host cost). Buffers, weight and group are captured by address and must
 * outlive the plan; runs of one plan, like calls on one weight, must not overlap. */
typedef struct j4b_qplan* j4b_qplan_t;
int j4b_quant_matvec_host_plan(j4b_qweight_t w, const float* x, int64_t batch, float* y, j4b_peer_group* g,
                               int channel, j4b_qplan_t* out);
int j4b_quant_matvec_host_run(j4b_qplan_t plan, j4b_stream s);
int j4b_quant_matvec_host_plan_free(j4b_qplan_t plan);
/* out[i] = sum over ranks of src[i], summed in rank order (identical on every rank). Both
 * collectives move 8-byte flagged words (value + step flag): a channel's slice of `bytes` holds
 * two parity halves, so a gathered output (batch * rows * nranks floats) or an all-reduce
 * (n * nranks floats) may take up to (bytes - 131072) / 16 / 16 words. */
int j4b_peer_allreduce(j4b_peer_group* g, int channel, j4b_buf src, int64_t n, j4b_buf out,
                       j4b_stream s);

/* ---- Decoder block (the Llama-style block of the quantised workloads; no reference counterpart:
 * the reference has no attention op, RoPE or KV cache, so a block written with its Tensor API
 * composes matmul, elementwise ops and axis reductions, and these kernels compute the same
 * functions). Activations are token-major f32 [tokens, width]. The fused QKV projection output
 * is [tokens, 3 * heads * head_dim] (q | k | v). The KV cache is f16 [batch, heads, capacity,
 * head_dim]; rotated queries are f32 [batch, heads, seq, head_dim]; attention output is token-
 * major f32 [batch * seq, heads * head_dim]. head_dim must be 128. ---- */
/* out[r, :] = x[r, :] / sqrt(mean(x[r, :]^2) + eps) * g; cols % 4 == 0, 16-byte aligned. */
int j4b_rmsnorm(j4b_buf x, j4b_buf g, float eps, int64_t rows, int64_t cols, j4b_buf out, j4b_stream s);
/* RoPE on q and k of tokens (b, t) at positions pos0 + t, t < seq: adjacent pairs (2i, 2i+1) of a
 * head rotated by pos * theta^(-2i / head_dim). Writes q_out, and k (rotated) and v as f16 into
 * the caches at slots pos0 .. pos0 + seq - 1. */
int j4b_rope_kv(j4b_buf qkv, int64_t batch, int64_t seq, int64_t heads, int64_t head_dim, int64_t pos0,
                double theta, j4b_buf q_out, j4b_buf k_cache, j4b_buf v_cache, int64_t capacity, j4b_stream s);
/* Decode: one query per sequence (q_out of j4b_rope_kv with seq 1) against the first `length`
 * cached tokens; out [batch, heads * head_dim]. f32 softmax and accumulation. */
int j4b_attention_decode(j4b_buf q, j4b_buf k_cache, j4b_buf v_cache, int64_t batch, int64_t heads,
                         int64_t head_dim, int64_t capacity, int64_t length, j4b_buf out, j4b_stream s);
/* Causal prefill of seq tokens per sequence (seq % 64 == 0, cached at slots 0 .. seq - 1): f16
 * tensor-core products with f32 softmax and accumulation (the rel 1e-2 tensor-core bar). */
int j4b_attention_prefill(j4b_buf q, j4b_buf k_cache, j4b_buf v_cache, int64_t batch, int64_t heads,
                          int64_t head_dim, int64_t capacity, int64_t seq, j4b_buf out, j4b_stream s);
/* out [rows, width] = gate * sigmoid(gate) * up, gate_up [rows, 2 * width] = gate | up. */
int j4b_swiglu(j4b_buf gate_up, int64_t rows, int64_t width, j4b_buf out, j4b_stream s);

/* ---- JIT tapes: ExecutionPlan.capture / execute (core/tensor/ExecutionPlan.java:49-132) ----
 *
 * A tape is the SPI call list a compiled function records once per input signature
 * (Jit.compile / compileTree, core/tensor/Jit.java:67-114), serialised as int64 words:
 *   header   MAGIC 0x314550415442344A, n_buffers, n_inputs, n_outputs, n_calls
 *   buffers  per buffer: rank, dims...
 *   inputs   buffer ids;  outputs  buffer ids
 *   calls    per call: opcode, out id, n_in, in ids..., n_attr, attrs...
 * Opcodes: 1 full, 2 fused, 3 transpose, 4 matmul, 5 batchedMatmul, 6 sliceAxis0, 7 stackAxis0,
 * 8 reduceSum, 9 reduceMax, 10 sumAxis, 11 maxAxis, 12 argMaxAxis, 13 maxAxisBackward,
 * 14 reshape, 15 broadcastTo, 16 reindex, 17 scatterAdd, 18 reluBackward, 19 randomUniform,
 * 20 randomNormal, 21 binary, 22 scalar, 23 unary. Attributes: full [value as f64 bits];
 * fused [postfix program: 0 idx | 1 op | 2 op | 3 op lo32 hi32]; sliceAxis0 [index];
 * sumAxis/maxAxis [axis, keep]; argMaxAxis/maxAxisBackward [axis]; reindex/scatterAdd
 * [1, offset, rank, strides...] (affine over the gather side's index) or [0, n, map...];
 * random [seed, counter]; binary/unary [op]; scalar [op, value as f64 bits].
 *
 * j4b_tape_compile validates the tape (J4B_EINVAL with the reference's messages), groups its
 * calls into fused sm_100a kernels (NVRTC) and allocates the tape's arena on `dev`.
 * j4b_tape_launch replays it: inputs and outputs are caller buffers (16-byte aligned, dense
 * f32, shapes as recorded; outputs must not alias inputs). Launches of one tape are serialised
 * by the tape (its arena is reused), as Jit.Compiled.apply is synchronized (Jit.java:80). */
typedef struct j4b_tape j4b_tape;
typedef struct j4b_tape_stats {
  int calls;          /* recorded SPI calls */
  int groups;         /* fused kernels */
  int folds;          /* cross-row reduction folds */
  int eager_steps;    /* calls run by the eager SPI kernels (matmul, transpose, ...) */
  int fills;
  int copies;
  int launches;       /* kernel launches per replay */
  int64_t arena_bytes;
} j4b_tape_stats;
int j4b_tape_compile(int dev, const int64_t* words, size_t nwords, j4b_tape** out);
int j4b_tape_launch(j4b_tape* tape, const j4b_buf* inputs, int n_inputs, const j4b_buf* outputs,
                    int n_outputs, j4b_stream s);
int j4b_tape_free(j4b_tape* tape);
int j4b_tape_info(j4b_tape* tape, j4b_tape_stats* stats);
/* Plans a tape and compiles its kernels without a device (NVRTC only): stats and the generated
 * CUDA source of every group. For tests and tooling on machines without a GPU. */
int j4b_tape_dryrun(const int64_t* words, size_t nwords, j4b_tape_stats* stats, char* buf,
                    size_t cap, size_t* len);
/* The generated CUDA source of fused kernel `group` (diagnostics). */
int j4b_tape_source(j4b_tape* tape, int group, char* buf, size_t cap, size_t* len);

/* ---- Scalar-AAD Monte-Carlo replay engines: AadEngine / AadExecutable
 * (core/engine/AadEngine.java:29-75, AadExecutable.java:34-75; the CUDA engines of
 * engine/CudaAadEngine.java, CudaInterpEngine.java, CudaEagerEngine.java).
 *
 * A tape is n_nodes records (ops[i], arg_a[i], arg_b[i], constants[i]) with op codes the AadOp
 * ordinals: 0 CONST, 1 INPUT (arg_a = input index), 2 RANDN (arg_a = draw ordinal, arg_b =
 * stream), 3 RANDU, 4 ADD, 5 SUB, 6 MUL, 7 DIV, 8 NEG, 9 EXP, 10 LOG, 11 SQRT, 12 MAX, 13 MIN,
 * 14 ABS; arguments name earlier nodes. input_nodes[j] is the INPUT node of input j and
 * output_node the single output. RANDU and named streams return J4B_EUNSUPPORTED, as the
 * reference's CUDA engines decline them (AadEngine.requireBasicRandom).
 *
 * engine: J4B_AAD_ENGINE_GENERATED ("cuda": per-tape generated kernel, NVRTC), _INTERP
 * ("cuda-interp": fixed interpreter kernel; at most 32 inputs), _EAGER ("cuda-eager": one launch
 * per node). precision: 4 = FLOAT32, 8 = FLOAT64 working precision; accumulation is always f64.
 * scratch_option: 0 = default; interpreter: threads; eager: scratch budget in bytes.
 *
 * A replay of `paths` scenarios starting at `path_offset` (scenario p draws from Philox keyed on
 * (p, seed), core/engine/cpu/Philox.java) produces sums[0] = sum of the output, sums[1] = sum of
 * its square and, with adjoints, sums[2 + j] = sum of d output / d input j. j4b_aad_replay takes
 * host inputs and returns host sums (blocking); j4b_aad_launch takes device inputs and sums and
 * is stream-ordered. A handle is not safe for concurrent use. */
#define J4B_AAD_ENGINE_GENERATED 0
#define J4B_AAD_ENGINE_INTERP 1
#define J4B_AAD_ENGINE_EAGER 2
typedef struct j4b_aad* j4b_aad_t;
int j4b_aad_compile(int dev, int engine, int n_nodes, const int32_t* ops, const int32_t* arg_a,
                    const int32_t* arg_b, const double* constants, int n_inputs,
                    const int32_t* input_nodes, int output_node, int precision, int adjoints,
                    int64_t scratch_option, j4b_aad_t* out);
int j4b_aad_replay(j4b_aad_t h, const double* inputs, uint64_t paths, uint64_t path_offset,
                   uint64_t seed, double* sums, j4b_stream s);
int j4b_aad_launch(j4b_aad_t h, j4b_buf inputs, uint64_t paths, uint64_t path_offset, uint64_t seed,
                   j4b_buf sums, j4b_stream s);
/* channels = 2 + inputs (with adjoints) or 2; compile_seconds of the generated kernel (0 for a
 * cached source and the fixed kernels); threads_or_slot: resident threads (generated),
 * interpreter threads, or eager scenarios per chunk. */
int j4b_aad_info(j4b_aad_t h, int* channels, double* compile_seconds, int64_t* threads_or_slot);
/* The generated kernel's CUDA source (empty for the interpreter and eager engines). */
int j4b_aad_source(j4b_aad_t h, char* buf, size_t cap, size_t* len);
int j4b_aad_free(j4b_aad_t h);
/* Validates a tape, generates its kernel source and compiles it with NVRTC, without a device. */
int j4b_aad_dryrun(int n_nodes, const int32_t* ops, const int32_t* arg_a, const int32_t* arg_b,
                   const double* constants, int n_inputs, const int32_t* input_nodes, int output_node,
                   int precision, int adjoints, char* buf, size_t cap, size_t* len);

#ifdef __cplusplus
}
#endif
#endif
