/*
 * zilla_b200.h -- C-ABI of libzilla_b200.so, the B200 (sm_100a) backend for
 * ZillaPHP's training hot path.
 *
 * Part 1 declares, with byte-identical signatures, every function that
 * ZillaPHP's CudaBackend binds through PHP FFI
 * (src/Hardware/CUDA/CudaBackend.php:51-95), so an FFI::cdef of that block
 * resolves against this library unchanged.  Part 2 adds entry points the
 * reference does not have (Adam, the fused training step, the data-parallel
 * runner, error reporting); they are additive and the reference's cdef
 * block does not need them.
 *
 * Conventions (kept from the reference):
 *   - Device memory lives in a handle registry (native/cuda/buffer_registry.cu:
 *     20-128): slots 1..8191, lowest free slot reused, 4-byte elements.
 *     Argmax indices (int32) and class targets (float-coded) share the
 *     float buffer type, as native/cuda/pooling_batched.cu:69 and
 *     native/cuda/training_ops.cu:7-9 do.
 *   - int-returning functions return 0 on success, -1 on an invalid handle,
 *     failed allocation or upload/download beyond capacity (as the reference),
 *     -2 on invalid sizes/arguments, -3 when a CUDA launch or call failed
 *     (the reference never reports launch failures; this library does).
 *   - All *_dev work is enqueued on one library stream per device; upload and
 *     download are synchronous with respect to it, so a download returns
 *     finished data (native/cuda/buffer_registry.cu:88,107).
 *   - Single-threaded caller (PHP); the registry is not thread-safe.
 */
#ifndef ZILLA_B200_H
#define ZILLA_B200_H

#ifdef __cplusplus
extern "C" {
#endif

/* ===================================================================== *
 * Part 1 -- the reference's CUDA C-ABI
 * ===================================================================== */

/* ---- host-pointer helpers (PCIe round trip per call) ---- */
/* native/cuda/matmul.cu:93-144: C[M,N] = A[M,K] @ B[K,N], row-major host arrays. */
void matmul_f32(const float *A, const float *B, float *C, int M, int K, int N);
/* native/cuda/elementwise.cu:71-148: elementwise ops on host arrays. */
void relu_f32_cuda(const float *X, float *Y, int N);
void add_f32_cuda(const float *A, const float *B, float *C, int N);
void sub_f32_cuda(const float *A, const float *B, float *C, int N);
void mul_f32_cuda(const float *A, const float *B, float *C, int N);
void div_f32_cuda(const float *A, const float *B, float *C, int N);
/* native/cuda/audio.cu:31-39: periodic-free Hann window 0.5-0.5cos(2 pi i/(N-1)). */
void hann_window_cuda(float *w, int N);
/* native/cuda/audio.cu:125-188: |rFFT| of Hann-windowed frames, output [nBins, nFrames].
 * Audio preprocessing, off the training path; kept so the reference's cdef resolves. */
void stft_magnitude_cuda(const float *input, int inputLen, const float *window, int fftSize,
                         int hopSize, float *output, int *outNBins, int *outNFrames);

/* ---- persistent buffer registry: native/cuda/buffer_registry.cu:39-128 ---- */
int zilla_buffer_alloc(unsigned long n_floats);
void zilla_buffer_free(int id);
int zilla_buffer_upload(int id, const float *host, unsigned long n_floats);
int zilla_buffer_download(int id, float *host, unsigned long n_floats);
void zilla_sync(void);
float *zilla_buffer_ptr(int id);

/* ---- device ops: native/cuda/device_ops.cu:44-149 ---- */
int matmul_dev(int a_id, int b_id, int c_id, int M, int K, int N);   /* C = A @ B */
int add_dev(int a_id, int b_id, int c_id, int n);
int sub_dev(int a_id, int b_id, int c_id, int n);
int mul_dev(int a_id, int b_id, int c_id, int n);
int div_dev(int a_id, int b_id, int c_id, int n);
int relu_dev(int x_id, int y_id, int n);

/* ---- training ops: native/cuda/training_ops.cu:42-288 ---- */
int add_bias_dev(int x_id, int b_id, int B, int C);                 /* :42-56   X[i,c] += b[c] */
int relu_fwd_dev(int x_id, int y_id, int mask_id, int n);           /* :62-78   y, float mask */
int relu_bwd_dev(int dy_id, int mask_id, int dx_id, int n);         /* :84-98   dx = dy*mask */
int softmax_ce_dev(int logits_id, int targets_id, int dlogits_id,   /* :110-163 loss += sum -log p_t */
                   int loss_id, int B, int C);                      /*          dZ = (p-onehot)/B  */
int bias_grad_dev(int dy_id, int db_id, int B, int C);              /* :169-184 db = column sums  */
int sgd_update_dev(int w_id, int dw_id, float lr, int n);           /* :190-203 W -= lr dW        */
int zero_dev(int id, int n);                                        /* :209-220 */
int matmul_tn_dev(int a_id, int b_id, int c_id, int M, int K, int N); /* :233-251 C = A^T B, A [K,M] */
int matmul_nt_dev(int a_id, int b_id, int c_id, int M, int K, int N); /* :258-276 C = A B^T, B [N,K] */
int copy_dev(int src_id, int dst_id, int n);                        /* :282-288 */

/* ---- per-sample conv / pool: native/cuda/conv2d.cu:71-259, native/cuda/pooling.cu:67-124 ---- */
int conv2d_fwd_dev(int input_id, int weight_id, int bias_id, int output_id, int C, int H, int W,
                   int outC, int outH, int outW, int kH, int kW, int stride, int padding);
int conv2d_bwd_dev(int input_id, int weight_id, int gradOut_id, int gradInput_id,
                   int gradWeight_id, int gradBias_id, int C, int H, int W, int outC, int outH,
                   int outW, int kH, int kW, int stride, int padding);
int maxpool2d_fwd_dev(int input_id, int output_id, int argmax_id, int C, int H, int W,
                      int outH, int outW, int kH, int kW, int stride);
int maxpool2d_bwd_dev(int gradOut_id, int argmax_id, int gradInput_id, int C, int outH, int outW);

/* ---- batched conv / pool: native/cuda/conv2d_batched.cu:69-271,
 *      native/cuda/pooling_batched.cu:61-116 ---- */
int conv2d_batched_fwd_dev(int input_id, int weight_id, int bias_id, int output_id, int B, int C,
                           int H, int W, int outC, int outH, int outW, int kH, int kW, int stride,
                           int padding);
int conv2d_batched_bwd_dev(int input_id, int weight_id, int gradOut_id, int gradInput_id,
                           int gradWeight_id, int gradBias_id, int B, int C, int H, int W,
                           int outC, int outH, int outW, int kH, int kW, int stride, int padding);
int maxpool2d_batched_fwd_dev(int input_id, int output_id, int argmax_id, int B, int C, int H,
                              int W, int outH, int outW, int kH, int kW, int stride);
int maxpool2d_batched_bwd_dev(int gradOut_id, int argmax_id, int gradInput_id, int B, int C,
                              int outH, int outW);

/* ---- attention primitives: native/cuda/attention.cu:83-251 ---- */
int softmax_rows_fwd_dev(int x_id, int y_id, int N, int M);
int softmax_rows_bwd_dev(int P_id, int dP_id, int dS_id, int N, int M);
int causal_mask_dev(int x_id, int N, int M, float maskValue);
int scale_dev(int x_id, float s, int n);
int causal_softmax_dev(int x_id, int N, int M, float maskValue);

/* ===================================================================== *
 * Part 2 -- additive entry points (no counterpart in the reference's cdef)
 * ===================================================================== */

/* Last error of this library as text ("" when none); the code of the last
 * failing call.  The reference only prints to stderr. */
const char *zilla_last_error(void);
int zilla_last_status(void);
/* Use the given cudaStream_t (as void*) for all following device work;
 * NULL restores the library's own stream. */
int zilla_set_stream(void *stream);
/* Number of kernel launches this library issued so far (instrumentation). */
unsigned long long zilla_launch_count(void);
/* Synchronises the library stream and reports (then clears) a kernel-side
 * error: -3 when a kernel skipped an out-of-range index (e.g. an argmax
 * outside dX in maxpool2d_*_bwd_dev) or a bounded wait expired, else 0. */
int zilla_check_device(void);

/* Adam (src/Optim/Adam.php:36-62) over one flat tensor of n floats, fused in
 * one kernel: m = b1 m + (1-b1) g; v = b2 v + (1-b2) g^2;
 * w -= lr (m/(1-b1^t)) / (sqrt(v/(1-b2^t)) + eps).  t is the 1-based step.
 * The reference has no native Adam (it runs in PHP). */
int adam_update_dev(int w_id, int g_id, int m_id, int v_id, float lr, float beta1, float beta2,
                    float eps, int t, int n);

/* The loss of the PHP CrossEntropy (src/Loss/CrossEntropy.php:56-59), which
 * clamps each row's target probability at 1e-12 before the log: loss +=
 * sum_rows -log(max(p_t, 1e-12)).  dlogits = (p - onehot)/B as softmax_ce_dev.
 * The native softmax_ce_dev has no clamp; this serves the Tensor / autograd
 * layer, whose rows can reach p_t < 1e-12 (a logit gap above 27.6). */
int softmax_ce_clamped_dev(int logits_id, int targets_id, int dlogits_id, int loss_id, int B, int C);

/* softmax_ce_dev for callers that cannot let a library allocate device memory
 * (code under a caller-owned memory pool or budget, or a host that only hands
 * over device pointers it already owns).  No counterpart in the reference.
 * Same arithmetic and the same outputs as softmax_ce_dev, on raw device
 * pointers and the caller's stream.  NULL means the library's own stream (the
 * one every *_dev op and zilla_set_stream use), so the call is ordered after
 * the ops that produced the logits; with any other stream the caller orders
 * it against the library's work (an event, or zilla_sync).  dlogits
 * = (softmax - onehot)/B, and the loss SUM over the rows is ADDED to *loss (the
 * caller zeroes it).  It calls no cudaMalloc, cudaFree or allocating library
 * routine: its per-row scratch is a file-scope static device array of 65536
 * doubles (512 KB on every GPU that loads the library, held until exit), so
 * B > 65536 is rejected with -2.  The first call on a device does the
 * set-up: it looks the array's device address up with cudaGetSymbolAddress,
 * so make that first call on each device before any stream capture.  All
 * calls share the array: calls that overlap on the GPU (other streams, other
 * host threads) race and must be serialised by the caller. */
int softmax_ce_noalloc(const float *logits, const float *targets, float *dlogits, float *loss,
                       int B, int C, void *stream);

/* ---- fused training step (replaces the ~30 per-op FFI calls of
 *      examples/mnist_cnn_gpu_v2.php:183-264 with one call) ----
 *
 * A "net" is a Sequential of layers given as int[4] rows {kind, a, b, c}:
 *   1 Conv2D 3x3 stride 1 (a = in channels, b = out channels, c = padding)
 *   2 ReLU
 *   3 MaxPool2D 2x2 stride 2
 *   4 Linear (a = in features, b = out features; W stored [in, out] as
 *     src/NN/Layers/Linear.php:14)
 * followed by softmax cross-entropy on the last layer's output.
 * Parameters are one flat float buffer in Sequential::parameters() order
 * (src/NN/Sequential.php:32-39): [W, b] per Conv2D/Linear layer, Conv2D W
 * in [outC, inC, 3, 3] (src/NN/Layers/Conv2D.php:25-44).
 *
 * precision: 0 = fp32 CUDA-core kernels everywhere (matches the reference
 *            within 1e-4 normwise);
 *            1 = bf16 tcgen05 tensor cores with fp32 accumulation for the
 *            dense conv and Linear contractions, fp32 master weights and
 *            fp32 optimizer state (larger, stated tolerance).
 * Returns a net id > 0, or a negative status. */
int zilla_net_create(const int *layers, int n_layers, int batch, int in_c, int in_h, int in_w,
                     int precision);
int zilla_net_destroy(int net);
/* Number of floats in the flat parameter buffer. */
long zilla_net_param_count(int net);
/* Registry handles of the flat parameter and gradient buffers (persistent
 * device tensors owned by the net; do not free). */
int zilla_net_params_id(int net);
int zilla_net_grads_id(int net);
/* Registry handle of the int32 argmax (global flat index, GPU batched
 * convention of native/cuda/pooling_batched.cu:39-52) of layer `layer`
 * (a MaxPool2D layer), materialised on request; 0 if unavailable. */
int zilla_net_argmax_id(int net, int layer);
/* Set optimizer: 1 = SGD (lr), 2 = Adam (lr, beta1, beta2, eps). */
int zilla_net_set_optimizer(int net, int kind, float lr, float beta1, float beta2, float eps);
/* One training step on device-resident inputs: x_id [batch, in_c*in_h*in_w],
 * y_id [batch] float-coded labels.  Writes the softmax_ce loss SUM over the
 * batch into loss_id[0] (softmax_ce_dev semantics, loss zeroed first),
 * leaves gradients in the grads buffer and updates the parameters.
 * update = 0 computes gradients only. */
int zilla_net_step(int net, int x_id, int y_id, int loss_id, int update);
/* Evaluation (forward pass only, the same kernels as the step's forward):
 * logits [batch, classes] fp32 into logits_id and, when y_id > 0 and
 * loss_id > 0, the softmax_ce loss SUM into loss_id[0].  No gradients, no
 * update.  Replaces the forward-only use of the layer stack in the
 * reference's evaluation loops (examples/mnist_cnn_gpu_v2.php:284-373);
 * not available for the language model (-2). */
int zilla_net_forward(int net, int x_id, int y_id, int logits_id, int loss_id);
/* Same step from host arrays: copies x/y host->device, runs the step and
 * copies the loss sum back (the end-to-end path). */
int zilla_net_step_host(int net, const float *x, const float *y, float *loss_sum, int update);
/* Staged host steps: the copy of the next batch runs during the current step.
 * No reference counterpart (additive; the reference copies each batch with a
 * blocking bufferUpload before its step, examples/mnist_cnn_gpu_v2.php:166-181).
 * zilla_net_stage_host enqueues the host->device copy of x and y into the
 * next of two device staging slots on the net's copy stream and returns at
 * once (host memory should be pinned for the copy to be asynchronous; it must
 * stay unchanged until the step that consumes it returns).  -2 when both
 * slots already hold batches not yet stepped.
 * zilla_net_step_staged runs the step on the oldest staged batch (-2 if none)
 * and, when loss_sum is not null, returns after copying the loss sum back.
 * Typical loop: stage(0); for k: stage(k+1); step_staged(k). */
int zilla_net_stage_host(int net, const float *x, const float *y);
int zilla_net_step_staged(int net, float *loss_sum, int update);
/* The staged step with a deferred loss read (no reference counterpart; the
 * reference's Trainer::fitLoader reads each step's loss with a blocking
 * item(), src/Training/Trainer.php:74-98).  zilla_net_step_staged_deferred
 * runs the step on the oldest staged batch and enqueues the copy of its loss
 * sum into pinned host memory, then waits only for the PREVIOUS deferred
 * step: that step's loss sum goes to *prev_loss_sum with *has_prev = 1 (0 on
 * the first call, or after a flush), while this step stays queued on the GPU.
 * zilla_net_loss_flush waits for the last deferred step and returns its loss
 * (*has = 0 when none is pending).  Typical loop: stage(0); for k: stage(k+1);
 * step_staged_deferred(k) -> loss of k-1; after the loop, flush -> last loss. */
int zilla_net_step_staged_deferred(int net, float *prev_loss_sum, int *has_prev, int update);
int zilla_net_loss_flush(int net, float *loss_sum, int *has);

/* Checkpoints: the net's parameters as a SafeTensors F32 file in the layout
 * ModelSerializer::save writes through SafeTensorsSerializer::save
 * (src/Serialization/ModelSerializer.php:56-69,
 * src/Serialization/SafeTensorsSerializer.php:32-98): u64 little-endian
 * header size, compact JSON header padded with spaces to 8 bytes, then the
 * data; one tensor "param_i" per parameter in Module::parameters() order with
 * its shape.  with_state != 0 also writes the Adam moments as "adam_m_i" /
 * "adam_v_i" and the step count as __metadata__ "adam_t" (the reference keeps
 * no optimizer state); it is rejected (-2) while the net is attached for
 * data parallelism over peer memory (each rank holds a slice of the state).
 * zilla_net_load reads such a file (or the reference's) into the net:
 * param_i required with matching shapes and dtype F32, adam_* optional;
 * -2 on a missing, malformed or mismatched file, and while the net is
 * attached for data parallelism over peer memory (detach, load the same file
 * on every rank, attach again). */
int zilla_net_save(int net, const char *path, int with_state);
int zilla_net_load(int net, const char *path);

/* Per-step CUDA graphs (no reference counterpart; the reference launches
 * about 30 FFI calls per step, examples/mnist_cnn_gpu_v2.php:183-264).
 * enable != 0: without profiling, the first step for given inputs (x, y
 * buffers and update flag) runs as is, the second is captured into a CUDA
 * graph and launched, later ones replay it with the optimizer's arguments of
 * the step; up to 16 input sets per net.  On one rank, or under the
 * peer-memory data-parallel step (one graph per input set and exchange
 * buffer, the exchange and update kernels given each step's number and Adam
 * arguments); the NCCL path runs plain.  Results are those of the plain step,
 * bit for bit.  zilla_net_set_optimizer, zilla_dp_attach and zilla_dp_detach
 * drop the graphs.  enable = 0 drops them and returns to plain launches. */
int zilla_net_set_graph(int net, int enable);

/* Device timing of the step's segments (instrumentation).  With profiling
 * enabled, zilla_net_step records a CUDA event after each kernel group;
 * zilla_net_timings then returns, for the last step, up to max_segments
 * durations in ms and their labels ('\n'-separated) and the segment count. */
int zilla_net_profile(int net, int enable);
/* Profiling of ONE segment: events only at the two boundaries of segment
 * `segment` (its index in zilla_net_timings' list of a fully profiled step),
 * so the step's other kernel boundaries carry no event.  zilla_net_timings
 * then returns that segment's duration once per step.  zilla_net_profile
 * (net, 0 or 1) ends it. */
int zilla_net_profile_segment(int net, int segment);
int zilla_net_timings(int net, char *labels, int labels_len, float *ms, int max_segments);
/* Diagnostics.  zilla_net_inspect returns the element count of the engine's
 * intermediate tensor `index` (0 past the last one), writes its name and,
 * when host != NULL, copies up to n_floats elements widened to float (bf16
 * activations, u8 pool codes).  Precision 1 only.  zilla_net_device_status
 * synchronises and reports a kernel-side error (a bounded wait that expired
 * or an index out of range) as -3 with the code in zilla_last_error(). */
int zilla_net_inspect(int net, int index, char *name, int name_len, float *host,
                      unsigned long n_floats);
int zilla_net_device_status(int net);

/* ---- fused Transformer language-model step (fp32) ----
 * Replaces TransformerLM::forwardBatch + the autograd backward + the
 * optimizer (src/Transformers/TransformerLM.php:77-116, trained as in
 * examples/train_shakespeare.php:104-124) with one call.  Pre-LN blocks
 * (src/Transformers/TransformerBlock.php:28-33): causal multi-head attention
 * (head dimension 32, src/Attention/MultiHeadAttention.php:41-80), FFN with
 * ReLU, LayerNorm eps 1e-5; final LayerNorm and Linear head; loss is
 * softmax_ce_dev's (sum over the batch*seq rows, gradients of the mean).
 * Parameters follow TransformerLM::parameters() (TransformerLM.php:158-170):
 * token table [vocab, dim], position table [max_seq, dim], final LN (g, b),
 * head (W [dim, vocab], b), then per block Wq bq Wk bk Wv bv Wo bo,
 * W1 [dim, ffn] b1, W2 [ffn, dim] b2, ln1 (g, b), ln2 (g, b).
 * The returned id is a net: zilla_net_set_optimizer / zilla_net_step /
 * zilla_net_step_host / zilla_net_params_id / zilla_dp_attach all apply,
 * with x = batch*seq token ids and y = batch*seq next-token ids, both as
 * floats.  seq <= 176 (one (sequence, head) of the attention backward is
 * held in shared memory).  Returns a net id > 0, or a negative status. */
int zilla_lm_create(int vocab, int dim, int heads, int layers, int max_seq, int ffn, int batch, int seq);
/* Generation with a K/V cache: TransformerLM::forwardWithCache
 * (src/Transformers/TransformerLM.php:124-151), as driven by
 * Sampler::generate (src/Generators/Sampler.php:35-100).  `count` token ids
 * (host floats, truncated like Embedding's (int) cast) take positions
 * len .. len+count-1, len = the cache length; each block appends their K and
 * V rows to its cache (MultiHeadAttention::forwardWithCache,
 * src/Attention/MultiHeadAttention.php:99-125) and every new row attends to
 * all cached rows WITHOUT a causal mask (attendHeadCached, :127-137).  logits
 * [count, vocab] fp32 are written to host memory (NULL skips the copy); the
 * cache length then grows by count.  len + count > max_seq or a token id
 * outside [0, vocab) returns kBadArg and leaves the cache unchanged (the
 * reference throws RuntimeException / OutOfRangeException).  Uses the net's
 * current parameters; independent of the training step's buffers. */
int zilla_lm_forward_cached(int net, const float *tokens, int count, float *logits);
/* Arithmetic of the language model's Linear layers (no reference counterpart;
 * the reference computes in float64 PHP): 0 = fp32 CUDA-core GEMMs (the
 * default; matches the reference within 1e-4), 1 = TF32 tcgen05 tensor-core
 * GEMMs for the blocks' Q/K/V, output, FFN projections and their input and
 * weight gradients (fp32 operands read with a 10-bit mantissa, fp32
 * accumulation; stated tolerance), with LayerNorm, attention, the head and
 * the loss unchanged.  Needs batch*seq % 256 == 0 and dim, ffn % 128 == 0. */
int zilla_lm_set_precision(int net, int precision);
/* TransformerLM::newCache (TransformerLM.php:153-156): cache length 0. */
int zilla_lm_cache_reset(int net);
/* KVCache::$length: the number of cached positions (>= 0), or a negative status. */
int zilla_lm_cache_length(int net);

/* ---- data-parallel runner (one process per GPU, NVLink) ----
 * zilla_dp_unique_id writes a 128-byte NCCL unique id (rank 0 creates it,
 * the host distributes it, e.g. through a file or a store).
 * zilla_dp_attach (collective) joins `net` to a communicator of `world`
 * ranks.  The per-rank batch is the net's batch; the global batch is world *
 * batch; gradients are scaled by 1/world before the update.  Two paths:
 *   bf16 engine, every GPU able to map every peer (ZB_PEER_STEP unset or not
 *   "0"): each rank owns a slice of the flat parameters; one kernel per step
 *   sums its slice of all ranks' gradients over NVLink peer memory, updates
 *   it and stores it into every rank's parameters.  After a step the
 *   parameters are identical on every rank, the loss slot holds the summed
 *   loss, and the gradient buffer holds the summed gradient of the rank's
 *   own slice only (the rest is this rank's local gradient).
 *   otherwise: the flat gradient buffer is summed with ncclAllReduce (the
 *   loss riding in it) and every rank runs the identical update.
 * zilla_dp_detach (collective) leaves the communicator; after a peer-memory
 * attach it first gives every rank the whole Adam state. */
int zilla_dp_unique_id(unsigned char *id128);
int zilla_dp_attach(int net, int rank, int world, const unsigned char *id128);
int zilla_dp_detach(int net);

#ifdef __cplusplus
}
#endif

#endif /* ZILLA_B200_H */
