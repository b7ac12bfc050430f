/*
 * b2e.h - C ABI of the B200 ensemble decode engine (libb2e.so).
 *
 * Plain C types only: pointers, sizes and status codes. Every function returns 0
 * on success or a negative B2E_ERR_* code; b2e_last_error() then holds a message
 * for the calling thread. Nothing here aborts, traps or prints.
 *
 * What each entry point replaces in the reference (huixu11/hackathon), whose hot
 * path is Python over torch:
 *   b2e_engine_create   NnInferenceClient.__init__: MultiTowerModel(config) +
 *                       load_state_dict + convert_linears + init_state(capacity)
 *                       (example_model.py:249-398)
 *   b2e_engine_step     one round of process_batch: stage features and the
 *                       active rows, run the step, read preds
 *                       (example_model.py:848-883, _step at :400-429)
 *   b2e_engine_reset_slots / read_slot / write_slot
 *                       init_state rows and the batched_state leaves
 *                       (model/inference_model.py:145-146)
 *   b2e_mlstm_step / b2e_retnet_step / b2e_mamba2_step
 *                       model/kernels.py mlstm_step / retnet_step / mamba2_step
 *                       (model/kernels.py:346-401)
 *   b2e_linear          CastLinear.forward / nn.Linear (example_model.py:92-95)
 *   b2e_layer_*         one layer's forward(x, state, mask) with its own state
 *                       table (model/xlstm.py:355, model/mamba2.py:62,
 *                       model/retnet.py:38, model/hawk.py:60)
 *   b2e_ingest_*        the client's request path up to process_batch:
 *                       ProtocolHandler.decode of each newline-delimited line
 *                       (protocol.py:86-103, SocketReader.read_all_available
 *                       :134-160), _handle_request's per-symbol queues
 *                       (client.py:156-173), _gather_requests (client.py:202-220)
 *                       and process_batch's rounds (example_model.py:885-899)
 *   b2e_encode_response ProtocolHandler.encode of an InferenceResponse
 *                       (protocol.py:80-84, protocol.py:38-44)
 */
#ifndef B2E_H
#define B2E_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B2E_API __attribute__((visibility("default")))
#else
#define B2E_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define B2E_OK 0
#define B2E_ERR_INVALID (-1)  /* bad argument, size or name */
#define B2E_ERR_CUDA (-2)     /* a CUDA runtime call failed */
#define B2E_ERR_WEIGHTS (-3)  /* weight missing, unexpected, or wrong size */
#define B2E_ERR_CAPACITY (-4) /* slot or batch outside the engine's capacity */
#define B2E_ERR_INTERNAL (-5)
#define B2E_ERR_DEVICE (-6)   /* a kernel recorded an error in the engine's device error word
                                 (a bounded wait timed out, or a device step got slots outside
                                 the table): that step's predictions and state are not valid.
                                 The word stays set, and every later b2e_engine_wait fails,
                                 until b2e_engine_device_error reads and clears it. */

/* Storage type of the nn.Linear weights: LINEAR_DTYPE of example_model.py:151-157.
 * The four fp32-kept linears (example_model.py:106), BlockLinear, convs and norms
 * stay float32 in every mode. */
#define B2E_FLAG_NO_PDL 1        /* launch chain kernels without programmatic dependent launch */
#define B2E_FLAG_NO_PRIORITIES 2 /* launch every chain at the same priority (default: the xLSTM tower's, the longest, first) */
#define B2E_FLAG_NO_LATENCY_PATH 4 /* run every host step through the batch graphs, never the one-kernel latency path */
#define B2E_FLAG_NO_PIPELINE 8 /* run each step as one graph whose four towers all finish before the next step starts
                                  (default: a tower's chain waits only for the same tower's previous step) */

#define B2E_DTYPE_F32 0
#define B2E_DTYPE_BF16 1
#define B2E_DTYPE_F16 2

/* Layer kinds, in MultiTowerModel's tower order (model/inference_model.py:107-112). */
#define B2E_LAYER_XLSTM 0
#define B2E_LAYER_MAMBA2 1
#define B2E_LAYER_RETNET 2
#define B2E_LAYER_HAWK 3

/* ModelConfig (model/inference_model.py:21-27) plus Mamba2's constructor sizes
 * (model/mamba2.py:10-17; the model uses head_size 64, bc_head_size 128). */
typedef struct b2e_model_config {
  int32_t hidden_size;
  int32_t proj_size;
  int32_t tower_depth;
  int32_t num_heads;
  int32_t num_features;
  int32_t mamba_head_size;
  int32_t mamba_bc_size;
} b2e_model_config;

typedef struct b2e_engine_options {
  int32_t device;       /* CUDA device ordinal */
  int32_t linear_dtype; /* B2E_DTYPE_* */
  int32_t capacity;     /* symbol slots of recurrent state (num_symbols, example_model.py:335) */
  int32_t max_batch;    /* rows per step, <= 65535 */
  int32_t use_graphs;   /* 1: replay each step from a CUDA graph per batch bucket */
  int32_t lanes;        /* independent row shares per tower for large batches; 0 = default (1) */
  int32_t lane_min_rows;/* batches from this many rows use `lanes`; 0 = default (256) */
  int32_t flags;        /* 0 = defaults; B2E_FLAG_NO_PDL turns PDL off, B2E_FLAG_NO_PRIORITIES priorities */
  int32_t lane_towers;  /* bit t set: tower t (0 xLSTM, 1 Mamba2, 2 RetNet, 3 Hawk) splits into `lanes`; 0 = every tower */
} b2e_engine_options;

/* A named float32 host tensor, keyed like MultiTowerModel.state_dict(). */
typedef struct b2e_tensor {
  const char* name;
  const float* data;
  int64_t numel;
} b2e_tensor;

typedef struct b2e_engine b2e_engine;
typedef struct b2e_layer b2e_layer;

B2E_API const char* b2e_last_error(void);
/* Grid of the state-streaming kernels (Mamba2 ssm, mLSTM C, RetNet S) when they
 * stream alone: b2e_mlstm_step / b2e_retnet_step / b2e_mamba2_step and the layer
 * engine. waves > 0 (default 8): short CTAs of a few items, ~waves waves of two
 * CTAs per SM; 0: one persistent CTA per SM, the grid the ensemble engine's step
 * always uses (its state kernels run beside the other towers' work). Results are
 * the same bit for bit; only the speed differs. Process-wide; *previous (may be
 * NULL) receives the old value. No counterpart in the reference. */
B2E_API int b2e_set_state_kernel_waves(int32_t waves, int32_t* previous);
B2E_API const char* b2e_version(void);

/* ---- ensemble engine (one per device) ---- */
B2E_API int b2e_engine_create(const b2e_model_config* cfg, const b2e_engine_options* opt, const b2e_tensor* tensors,
                      int32_t n_tensors, b2e_engine** out);
B2E_API void b2e_engine_destroy(b2e_engine* e);
/* One step over n rows: slots[n] (distinct, < capacity), features[n * num_features]
 * and preds[n * 4] are HOST buffers; columns are xLSTM, Mamba2, RetNet, Hawk. */
B2E_API int b2e_engine_step(b2e_engine* e, const int32_t* slots, const float* features, int32_t n, float* preds);
/* The same step split in two, so several devices run at once. Up to two submits
 * may be outstanding on one engine (wait returns the oldest step's
 * predictions): the second step's input copies and the first step's prediction
 * copies run beside the steps themselves. The engine's device error word is
 * copied back with the predictions: wait (and step) return B2E_ERR_DEVICE when
 * it is set. */
B2E_API int b2e_engine_submit(b2e_engine* e, const int32_t* slots, const float* features, int32_t n);
B2E_API int b2e_engine_wait(b2e_engine* e, float* preds);
/* Device-buffer step enqueued on `stream` (a cudaStream_t, NULL = default stream).
 * Slots outside the table step no row and set a flag read by b2e_engine_device_error. */
B2E_API int b2e_engine_step_device(b2e_engine* e, const int32_t* d_slots, const float* d_features, int32_t n,
                           float* d_preds, void* stream);
/* Device-buffer steps that overlap: each submit reads d_slots / d_features after
 * the work enqueued on `stream` so far and writes d_preds when its step ends, but
 * does not make `stream` wait for that end; b2e_engine_join_device(e, stream)
 * does, for every step submitted before it. Until the join the caller leaves
 * the step's three buffers alone. Consecutive steps are ordered per tower (a
 * tower's chain waits for the same tower's previous step), so one step's towers
 * run beside the next step's; results are those of the steps run one by one.
 * Refused while a host step (b2e_engine_submit) is in flight. No counterpart in
 * the reference, which steps one round at a time (example_model.py:848-883). */
B2E_API int b2e_engine_submit_device(b2e_engine* e, const int32_t* d_slots, const float* d_features, int32_t n,
                             float* d_preds, void* stream);
B2E_API int b2e_engine_join_device(b2e_engine* e, void* stream);
B2E_API int b2e_engine_device_error(b2e_engine* e, int32_t* flag);
B2E_API int b2e_engine_reset_slots(b2e_engine* e, const int32_t* slots, int32_t n);
/* One slot's whole state, every leaf in iter_state_tensors order
 * (example_model.py:160-176) and in the reference's per-row layout. */
B2E_API int b2e_engine_slot_bytes(const b2e_engine* e, int64_t* bytes);
B2E_API int b2e_engine_read_slot(b2e_engine* e, int32_t slot, void* host, int64_t bytes);
B2E_API int b2e_engine_write_slot(b2e_engine* e, int32_t slot, const void* host, int64_t bytes);
/* Kernels one step of n rows launches (counted from its captured graph; 1 when
 * the step runs on the latency path). */
B2E_API int b2e_engine_launches(b2e_engine* e, int32_t n, int32_t* kernels);
/* Host steps of at most *rows rows run as one kernel (one thread-block cluster
 * of *cluster CTAs per tower) instead of the batch graph; *rows = 0 when these
 * dims or this GPU keep every step on the graphs. The latency path behind
 * b2e_engine_step / submit; no counterpart in the reference (a property of this
 * engine, reported for tests and measurement). */
B2E_API int b2e_engine_latency_rows(b2e_engine* e, int32_t* rows, int32_t* cluster);
B2E_API int b2e_engine_memory(const b2e_engine* e, int64_t* weight_bytes, int64_t* state_bytes);

/* ---- fused state steps: the model/kernels.py operator API ----
 * All pointers are DEVICE pointers to contiguous float32 arrays; mask is a
 * device bool/uint8 array of `batch` entries or NULL (every row active). The
 * state is updated in place on active rows only; out gets zeros on idle rows. */
B2E_API int b2e_mlstm_step(float* cell, const float* q, const float* k, const float* v, const float* i_gate,
                   const float* f_gate, const uint8_t* mask, int32_t batch, int32_t heads, int32_t size_h,
                   int32_t size_k, float* out, void* stream);
B2E_API int b2e_retnet_step(float* state, const float* k_rope, const float* v, const float* q_scaled, const float* decay,
                    const uint8_t* mask, int32_t batch, int32_t heads, int32_t size_h, int32_t size_k, float* out,
                    void* stream);
B2E_API int b2e_mamba2_step(float* ssm, const float* x, const float* b, const float* c, const float* dt,
                    const float* decay, const uint8_t* mask, int32_t batch, int32_t heads, int32_t size_h,
                    int32_t size_c, float* out, void* stream);

/* ---- one projection: CastLinear.forward / nn.Linear ----
 * y[m, n] = act(round(sum_k x[m, k] * w[n, k] + bias[n])) in float32, where with
 * a low-precision weight (B2E_DTYPE_BF16/F16) x is rounded to that type first
 * and `round` rounds the result to it, as CastLinear does; with an f32 weight
 * there is no rounding. x has type x_dtype (f32 or the weight's type), bias the
 * weight's type; act 0 = none, 1 = ReLU. Device pointers; d_err is a device int
 * that receives an error code if the tensor-core kernel times out (NULL keeps
 * the problem off the tensor-core kernel). */
B2E_API int b2e_linear(const void* x, int32_t x_dtype, int32_t m, int32_t k, const void* w, int32_t w_dtype,
                       const void* bias, int32_t n, int32_t act, float* y, int32_t* d_err, void* stream);

/* ---- b2e_linear for callers that cannot allocate device memory ----
 * No counterpart in the reference: an addition of this library. Same operands,
 * types and result as b2e_linear, but every byte of scratch (the tensor-core
 * kernel's error word and, for an f32 x with a bf16/fp16 weight, x rounded to
 * the weight's type) lives in one static device array of 16 MiB + 256 B inside
 * the library, so the call makes no cudaMalloc, cudaFree or other allocating
 * call. For hosts whose device memory is all owned by their own pool, and for
 * loops that must not allocate after start-up.
 *  - f32 x with a bf16/fp16 weight needs m * k <= 8388608; larger is refused
 *    with B2E_ERR_INVALID (use b2e_linear).
 *  - The first call on a device (the current device) looks up the array's
 *    device address; make that first call before any stream capture.
 *  - Every GPU that loads the library holds the array until the process exits.
 *  - All calls share the array: calls that overlap on the GPU (other streams,
 *    other threads) race. Each call clears the error word it needs.
 *  - h_err: NULL, or a host int; when given, the call waits for the stream and
 *    stores there the tensor-core kernel's error code (0 = finished): this
 *    call's, or, when this call finished, a code that earlier calls made with
 *    h_err NULL left pending (kept in the array until a call reports it). */
B2E_API int b2e_linear_static(const void* x, int32_t x_dtype, int32_t m, int32_t k, const void* w,
                              int32_t w_dtype, const void* bias, int32_t n, int32_t act, float* y,
                              int32_t* h_err, void* stream);

/* ---- one recurrent layer with its own state table ----
 * Weights are keyed like that layer's own state_dict() (no prefix). */
B2E_API int b2e_layer_create(int32_t kind, const b2e_model_config* cfg, const b2e_engine_options* opt,
                     const b2e_tensor* tensors, int32_t n_tensors, b2e_layer** out);
B2E_API void b2e_layer_destroy(b2e_layer* l);
/* y[n, hidden] = layer(x[n, hidden]) for rows at d_slots[n]; device buffers. */
B2E_API int b2e_layer_step_device(b2e_layer* l, const int32_t* d_slots, const float* d_x, int32_t n, float* d_y,
                          void* stream);
B2E_API int b2e_layer_reset_slots(b2e_layer* l, const int32_t* slots, int32_t n);
B2E_API int b2e_layer_slot_bytes(const b2e_layer* l, int64_t* bytes);
B2E_API int b2e_layer_read_slot(b2e_layer* l, int32_t slot, void* host, int64_t bytes);
B2E_API int b2e_layer_write_slot(b2e_layer* l, int32_t slot, const void* host, int64_t bytes);

/* ---- request ingest (host only; no GPU needed) ----
 * Raw bytes from the server's socket go in; requests come out as flat arrays
 * (symbol ids, unique ids, float32 feature rows) in process_batch's round order,
 * with no per-request or per-float Python objects.
 *
 * b2e_ingest_feed splits the bytes into lines (a partial last line waits for
 * the next feed). A line that json.loads would read as an "inference_request"
 * message with exactly the fields of InferenceRequest (unique_ids: integers
 * within int64, symbols: ASCII-escaped strings, features: rows of num_features
 * numbers, timestamp: any value) is decoded natively: for i < min(len(unique_ids),
 * len(symbols), len(features)) request i is appended to its symbol's queue, or,
 * when that queue already holds max_queue requests, dropped and reported by
 * b2e_ingest_next_drop (client.py:169-173). Every other non-empty line (other
 * message types, malformed JSON, other field types, non-ASCII bytes) is kept
 * whole for the caller's own decoder (b2e_ingest_next_other), and the feed
 * stops right after it, so that what the caller does with it (a request it
 * queues with b2e_ingest_push) comes before the lines after it; feed again
 * (len 0 is fine) to go on.
 * Symbols get dense ids in order of first sight; that order is the order of the
 * reference's request_queues dict, so it is also process_batch's symbol order.
 * b2e_ingest_take drains every queue at once (_gather_requests) and writes the
 * rows round by round: round k holds the k-th queued request of every symbol
 * that has one, symbols in id order (example_model.py:885-899). Buffers hold at
 * least b2e_ingest_pending() rows (round_rows: that many entries). */
typedef struct b2e_ingest b2e_ingest;
B2E_API int b2e_ingest_create(int32_t num_features, int32_t max_queue, b2e_ingest** out);
B2E_API void b2e_ingest_destroy(b2e_ingest* g);
/* Threads that parse the lines of one feed side by side (default: up to 8, the
 * host's hardware threads); requests are still queued in line order. */
B2E_API int b2e_ingest_set_threads(b2e_ingest* g, int32_t threads);
B2E_API int b2e_ingest_feed(b2e_ingest* g, const char* data, int64_t len, int32_t* n_requests, int32_t* n_other);
/* The oldest kept line (without its newline); *len = -1 when there is none, or
 * the line's length when cap is too small (nothing is consumed then). */
B2E_API int b2e_ingest_next_other(b2e_ingest* g, char* buf, int64_t cap, int64_t* len);
/* Queue one request the caller decoded itself (symbol: UTF-8 bytes); *queued
 * = 0 when its symbol's queue was full (then reported as a drop). */
B2E_API int b2e_ingest_push(b2e_ingest* g, int64_t unique_id, const char* symbol, int64_t symbol_len,
                            const float* features, int32_t* queued);
/* Symbol id of the oldest dropped request, or -1 when there is none. */
B2E_API int b2e_ingest_next_drop(b2e_ingest* g, int32_t* symbol);
B2E_API int b2e_ingest_pending(const b2e_ingest* g, int64_t* rows);
B2E_API int b2e_ingest_symbol_count(const b2e_ingest* g, int32_t* n);
/* UTF-8 name of a symbol id; *len as in b2e_ingest_next_other. */
B2E_API int b2e_ingest_symbol_name(const b2e_ingest* g, int32_t symbol, char* buf, int64_t cap, int64_t* len);
B2E_API int b2e_ingest_take(b2e_ingest* g, int64_t cap, int32_t* symbols, int64_t* unique_ids, float* features,
                            int32_t* round_rows, int32_t* n_rounds, int64_t* n_rows);

/* One micro-batch for continuous batching: the oldest queued request of each of
 * up to max_rows distinct symbols, taken in the arrival order of those requests;
 * a symbol's later requests stay queued for later calls, so its requests are
 * still taken in order and at most once per batch. The request loop's
 * counterpart of b2e_ingest_take (client.py:202-220's drain and
 * example_model.py:885-899's rounds) for a caller that steps batches as they
 * form instead of waiting for a whole drain. */
B2E_API int b2e_ingest_take_batch(b2e_ingest* g, int32_t max_rows, int32_t* symbols, int64_t* unique_ids,
                                  float* features, int32_t* n_rows);

/* The bytes ProtocolHandler.encode(InferenceResponse(unique_ids, predictions,
 * client_timestamp)) produces: json.dumps' layout and float repr (predictions
 * widened float32 -> double as p.astype(float).tolist() does), newline
 * included. *len = bytes written, or the size needed when cap is too small. */
B2E_API int b2e_encode_response(const int64_t* unique_ids, const float* predictions, int64_t n, int32_t n_out,
                                double client_timestamp, char* buf, int64_t cap, int64_t* len);

#ifdef __cplusplus
}
#endif

#endif /* B2E_H */
