/*
 * cpde_b200 - C ABI of the B200-native cPDE engine.
 *
 * The reference's boundary for this path is the cpde_server wire protocol
 * (cuda/protocol.hpp:10-51, opcodes of cuda/cpde_server.cu:436-555). Each
 * entry point below replaces one opcode handler (cited on the declaration);
 * bin/cpde_server decodes frames and calls exactly these functions, so any
 * client of the reference server (its Python package included) drives this
 * engine unchanged. All arguments are plain pointers, sizes and integers.
 *
 * Conventions
 *  - Every function returns CPDE_OK, CPDE_REJECTED (the request was invalid;
 *    nothing changed and the engine stays usable; the reference answers such
 *    requests with a kind-1 reply) or CPDE_DEVICE_ERROR (a CUDA failure).
 *    cpde_last_error() returns the message of the last failure on that engine
 *    thread-safely with respect to the engine's single executor.
 *  - Object handles are the u64 ids of the reference (cuda/cpde_server.cu:98):
 *    data, networks and costs share one counter starting at 1.
 *  - Arrays use the reference's layouts: data values (derivative, sample,
 *    channel); weights per layer column-major W (n_l x n_{l-1}) then bias.
 *  - Variable-length results are delivered through a cpde_sink callback that
 *    is called exactly once per result before the function returns.
 */
#ifndef CPDE_B200_H
#define CPDE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct cpde_engine cpde_engine;

#define CPDE_OK 0
#define CPDE_REJECTED 1
#define CPDE_DEVICE_ERROR 2

/* Receives one byte range (a reply payload, a state blob, a source string). */
typedef void (*cpde_sink)(void* context, const void* bytes, size_t length);
/* Receives one wire event during training: kind 2/3/4/5/6 payloads exactly as
 * the reference streams them (cuda/cpde_server.cu:319-340,424,426), and the
 * final kind-0 result (u64 completed, i32 stopped, u8[] metadata). */
typedef void (*cpde_event_sink)(void* context, uint32_t kind, const void* payload, size_t length);

/* Creates an engine on one CUDA device. Replaces Server::Server(int) and the
 * `--device N` command line (cuda/cpde_server.cu:103,562). */
int cpde_engine_create(int32_t device, cpde_engine** engine);

/* Creates one rank of a point-sharded engine group: every rank holds its own
 * shard of each Data object and the weight gradients and cost totals of every
 * epoch are summed over ranks with one NCCL all-reduce before validation and
 * the optimizer update, so replicas stay identical. `unique_id` is the 128-byte
 * NCCL id from cpde_sharding_id() on rank 0, shared by the caller. New; the
 * reference is single-device (cuda/cpde_server.cu:562). */
int cpde_engine_create_sharded(int32_t device, int32_t rank, int32_t world, const void* unique_id,
                               cpde_engine** engine);
int cpde_sharding_id(void* unique_id, size_t capacity);
/* The contiguous sample range [lo, lo + count) that rank `rank` of `world`
 * holds of a Data object with `total` samples (remainder spread over the first
 * ranks). Host only; no device or engine needed. New. */
int cpde_shard_range(int64_t total, int32_t rank, int32_t world, int64_t* lo, int64_t* count);

void cpde_engine_destroy(cpde_engine* engine);
const char* cpde_last_error(const cpde_engine* engine);

/* Op 1 handshake: protocol "CPDE/3", version 6, capability bits
 * (cuda/cpde_server.cu:438-447). */
int cpde_hello(cpde_engine* engine, cpde_sink reply, void* context);

/* Op 2: create input or target data (cuda/cpde_server.cu:449-454). `table` is
 * derivatives x (variables+1) row-major (order, counts...); `values` has
 * derivatives*samples*channels floats. */
int cpde_data_create(cpde_engine* engine, int32_t derivatives, int32_t channels, int32_t samples,
                     int32_t variables, const int32_t* table, size_t table_count, const float* values,
                     size_t value_count, uint64_t* id);
/* Shape of a data object (derivatives, channels, samples). */
int cpde_data_shape(cpde_engine* engine, uint64_t id, int32_t* derivatives, int32_t* channels, int32_t* samples);
/* Op 5: download (cuda/cpde_server.cu:475). */
int cpde_data_download(cpde_engine* engine, uint64_t id, float* values, size_t count);
/* Op 6: replace the values and bump the version (cuda/cpde_server.cu:476). */
int cpde_data_replace(cpde_engine* engine, uint64_t id, const float* values, size_t count);

/* Op 3: create a network with its initial weights, one array per layer
 * (cuda/cpde_server.cu:455-473). `linear[i]` is 1 (linear), 0 (sigmoid) or,
 * as an extension, 2 (tanh). */
int cpde_net_create(cpde_engine* engine, const int32_t* neurons, const int32_t* linear, int32_t layers,
                    const float* const* initial, const size_t* initial_counts, uint64_t* id);
/* Op 4: evaluate every derivative row of `data` (cuda/cpde_server.cu:171-183). */
int cpde_net_evaluate(cpde_engine* engine, uint64_t net, uint64_t data, int32_t chunk, uint64_t* output);
/* Op 9: state blob (cuda/cpde_server.cu:193-206). */
int cpde_net_snapshot(cpde_engine* engine, uint64_t net, cpde_sink blob, void* context);
/* Op 10: restore a state blob (cuda/cpde_server.cu:207-222). */
int cpde_net_restore(cpde_engine* engine, uint64_t net, const void* blob, size_t length);

/* Op 7, kind 0: squared-error matching cost (cuda/cpde_server.cu:477-480). */
int cpde_cost_matching(cpde_engine* engine, uint64_t net, uint64_t inputs, uint64_t targets, int32_t chunk,
                       const int32_t* rows, size_t row_count, const int32_t* target_rows, size_t target_row_count,
                       int32_t weight_samples, const float* weights, size_t weight_count, uint64_t* id);
/* Op 7, kind 1: linear/quadratic polynomial residuals (cuda/cpde_server.cu:481).
 * `terms` holds (equation, a, b) triples. */
int cpde_cost_polynomial(cpde_engine* engine, uint64_t net, uint64_t inputs, int32_t chunk, const int32_t* rows,
                         size_t row_count, int32_t equations, const int32_t* terms, size_t term_words,
                         const float* coefficients, size_t coefficient_count, const float* rhs, size_t rhs_count,
                         const float* weights, size_t weight_count, uint64_t* id);
/* Op 12: compiled scalar integral over samples (cuda/cpde_server.cu:489-533).
 * `nodes` holds (op, a, b) triples of the scalar IR. */
int cpde_cost_integral(cpde_engine* engine, uint64_t net, uint64_t inputs, int32_t chunk, int32_t samples,
                       const int32_t* nodes, size_t node_words, const double* constants, size_t constant_count,
                       int32_t fields, const double* field_values, size_t field_count, const double* weights,
                       size_t weight_count, uint64_t* id);
/* Op 13: generated source and compile log of an integral cost, compiling it
 * first when `compile` is nonzero (cuda/cpde_server.cu:534). */
int cpde_cost_source(cpde_engine* engine, uint64_t cost, int32_t compile, cpde_sink code, cpde_sink log,
                     void* context);
/* Op 11: release data (kind 0), a network (1) or a cost (2)
 * (cuda/cpde_server.cu:486-488). */
int cpde_release(cpde_engine* engine, int32_t kind, uint64_t id);

/* Op 8 (graph_mode 0) and op 15 (graph_mode 1): training epochs. `request`
 * is the opcode's payload (cuda/cpde_server.cu:364-371); events stream
 * through `events` and end with the kind-0 result. `stop` (may be NULL) is
 * polled between updates: nonzero stops at the next update boundary, as
 * op 99 does (cuda/cpde_server.cu:566,384). */
int cpde_train(cpde_engine* engine, int32_t graph_mode, const void* request, size_t length, cpde_event_sink events,
               void* context, const volatile int32_t* stop);
/* Op 14: value of a cost graph and optionally its weight gradients at fixed
 * weights; optimizer state is unchanged (cuda/cpde_server.cu:535-551). */
int cpde_graph_evaluate(cpde_engine* engine, const void* request, size_t length, cpde_sink reply, void* context);
/* Op 90: benchmark epochs, reply f64[] wall ms, f64[] device ms, f64 loss,
 * f32[] gradient per layer (docs/benchmarks/fourier-timing.patch:13-35). */
int cpde_benchmark(cpde_engine* engine, uint64_t net, uint64_t cost, int32_t warm, int32_t iterations,
                   int32_t batches, cpde_sink reply, void* context);

/* --- Direct epoch control (no reference counterpart; used by benchmarks) --- */

/* Enqueues one fixed-weight epoch of `costs` (forward of every chunk, loss,
 * output adjoints, backward into the active gradient buffers) on the engine's
 * stream without synchronising; the body of op 90's timed step. */
int cpde_epoch(cpde_engine* engine, uint64_t net, const uint64_t* costs, size_t count);
/* Waits for the stream, then copies the summed objective and the flat
 * gradient of all layers (layer order, W then bias) to host memory. */
int cpde_epoch_result(cpde_engine* engine, uint64_t net, double* objective, float* gradient, size_t count);
/* The cudaStream_t every kernel of this engine is launched on. */
int cpde_engine_stream(cpde_engine* engine, void** stream);
/* Per-kernel device timing with CUDA events around each launch (off by
 * default). The report is text: one "name launches total_ms" line per kernel. */
int cpde_kernel_timing(cpde_engine* engine, int32_t enable);
int cpde_kernel_timing_report(cpde_engine* engine, cpde_sink report, void* context);
/* Selects the execution tier: 0 automatic, 1 generic kernels only, 2 tensor-core
 * (tcgen05 3xTF32) GEMMs wherever the layer shapes allow, 3 the single-launch
 * point-tile epoch wherever it applies (matching costs on the fused head), 4
 * the fused fast-tier kernels with exact-FP32 FFMA GEMMs only. No reference
 * counterpart. */
int cpde_set_tier(cpde_engine* engine, int32_t tier);

/* Weight gradient of one layer without any device allocation. No counterpart
 * in the reference. It serves callers that cannot call cudaMalloc: hosts whose
 * own allocator already owns the device memory (a framework's preallocated
 * pool leaves no room for a second allocator, and an allocation that fails in
 * the middle of their step cannot be recovered), and code on a latency-bound
 * path that must not take cudaMalloc's or cudaFree's implicit device
 * synchronisation. Computes gradient = dZ [A; 1]^T, an outputs x (inputs+1)
 * column-major matrix (weights, then the bias column = sum of dZ over the
 * value-row columns c with c % rows == 0), from device arrays in the
 * interleaved layout: column c = point*rows + row, `dz` outputs x
 * (points*rows), `activations` inputs x (points*rows), both 16-byte aligned,
 * outputs and inputs multiples of 4. Split partial sums live in a static
 * 16 MiB device array (4194304 floats, held by every GPU that loads the
 * library until exit); outputs*(inputs+1) beyond that is rejected. The first
 * call on a device looks up the array's device address once (with that device
 * current) and keeps it for the life of the process, so make that first call
 * before any stream capture, and do not call it again after resetting the
 * device (cudaDeviceReset), which invalidates the address. Calls are
 * asynchronous on `stream` (NULL: the engine's stream); calls that overlap on
 * the GPU race on the shared array. */
int cpde_layer_gradient_static(cpde_engine* engine, const float* dz, const float* activations, int32_t outputs,
                               int32_t inputs, int64_t points, int32_t rows, float* gradient, void* stream);

/* Host-only schema compiler (no device needed): Leibniz jet tables for the
 * given rows x variables count matrix, packed as documented in schema.hpp. */
int cpde_jet_plan(const int32_t* counts, int32_t rows, int32_t variables, int32_t* packed, size_t capacity,
                  size_t* length);

#ifdef __cplusplus
}
#endif

#endif /* CPDE_B200_H */
