/* sheaf_b200 executor C ABI.
 *
 * Drop-in replacement for the subset of the IREE runtime C API that Sheaf's
 * runtime binds (sheaf/src/runtime/iree_ffi.rs:149-297) to run compiled
 * fwd+VJP (`value_and_grad`) and forward modules. The semantics mirror IREE's
 * one-to-one so the Rust shim is a rename:
 *
 *   iree_runtime_instance_create + try_create_default_device
 *     + session_create_with_device        -> sb_session_create
 *   iree-compile + session_append_bytecode_module_from_memory
 *                                         -> sb_module_load_stablehlo
 *   iree_runtime_session_call_by_name     -> sb_call
 *   iree_hal_buffer_view_allocate_buffer_copy -> sb_buffer_alloc_copy
 *   iree_hal_device_transfer_d2h          -> sb_buffer_d2h
 *   iree_hal_buffer_view_{retain,release,shape_rank,shape_dim,element_type}
 *                                         -> sb_buffer_{retain,release,rank,dim,elem_type}
 *   iree_status_{is_ok,format,free}        -> sb_status_{is_ok,message,free}
 *
 * Status: NULL means OK; otherwise an owned object the caller frees.
 * Buffers are reference counted; a buffer keeps its session alive.
 * Calls are asynchronous on the session's stream: outputs are ready when
 * read (sb_buffer_d2h waits, with a bounded timeout).
 * Element types use IREE HAL codes (sheaf/src/runtime/iree_ffi.rs:32-36).
 */
#ifndef SHEAF_B200_H_
#define SHEAF_B200_H_

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#include "sheaf_b200_ops.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct sb_status_s* sb_status;
typedef struct sb_session_s sb_session;
typedef struct sb_buffer_s sb_buffer;
typedef struct sb_module_s sb_module;

/* Status codes (mirroring iree_status_code_t values where one exists). */
#define SB_STATUS_OK 0
#define SB_STATUS_INVALID_ARGUMENT 3
#define SB_STATUS_DEADLINE_EXCEEDED 4
#define SB_STATUS_NOT_FOUND 5
#define SB_STATUS_RESOURCE_EXHAUSTED 8
#define SB_STATUS_FAILED_PRECONDITION 9
#define SB_STATUS_UNIMPLEMENTED 12
#define SB_STATUS_INTERNAL 13
#define SB_STATUS_UNAVAILABLE 14

/* ---- status (replaces iree_status_*, iree_ffi.rs:145-147,281-288) ---- */
SB_API bool sb_status_is_ok(sb_status status);
SB_API int sb_status_code(sb_status status);
SB_API const char* sb_status_message(sb_status status);
SB_API void sb_status_free(sb_status status);

/* ---- session (replaces IreeSession::new, iree_session.rs:122-231) ---- */
/* One session per process per GPU. The device must be an sm_100 part. */
SB_API sb_status sb_session_create(int device_ordinal, sb_session** out_session);
SB_API void sb_session_retain(sb_session* session);
SB_API void sb_session_release(sb_session* session);
/* Waits for all work queued on the session; DEADLINE_EXCEEDED after timeout_ns
 * (< 0 = no limit). Also reports a kernel-side bounded-wait timeout. */
SB_API sb_status sb_session_synchronize(sb_session* session, int64_t timeout_ns);
/* The session's cudaStream_t (for callers that interleave their own work). */
SB_API void* sb_session_stream(sb_session* session);
/* Dispatch counters in the spirit of `--jit-profile`
 * (sheaf/src/runtime/iree_session.rs:250-297). kernel_launches counts every
 * library kernel the session's calls have launched (kernel nodes of a
 * replayed CUDA graph included). */
typedef struct sb_session_stats {
  uint64_t calls;
  uint64_t graph_captures;
  uint64_t graph_replays;
  uint64_t kernel_launches;
} sb_session_stats;
SB_API sb_status sb_session_get_stats(sb_session* session, sb_session_stats* out_stats);

/* ---- data-parallel group (no reference counterpart: roadmap item
 * "NCCL all-reduce", docs/roadmap.md:61-62) ----
 * Joins this session to an NCCL group of `world` ranks. Afterwards every
 * value_and_grad call all-reduces (averages) the loss and the gradients, each
 * rank having received its own equal batch shard. */
#define SB_NCCL_ID_BYTES 128
SB_API sb_status sb_nccl_unique_id(void* out_id, size_t id_bytes);
SB_API sb_status sb_session_join_group(sb_session* session, const void* nccl_id, size_t id_bytes, int rank, int world);
/* Leaves the group; later calls run on this rank's data alone. Call it only
 * between steps, with none of this session's collectives in flight: an
 * enqueued all-reduce waits on the GPU for every peer without a limit. With
 * `abort` non-zero the communicator is ended with ncclCommAbort (for the
 * survivors of a rank that has left: nothing waits for the missing peer);
 * otherwise with ncclCommDestroy. */
SB_API sb_status sb_session_leave_group(sb_session* session, int abort);

/* ---- buffers (replaces buffer_convert.rs:14-123, device_buffer.rs:47-134) ---- */
/* Allocates a device buffer from the session pool and copies `bytes` of host
 * data into it (bytes must equal the element count times the element size). */
SB_API sb_status sb_buffer_alloc_copy(sb_session* session, const int64_t* shape, size_t rank, uint32_t elem_type,
                                      const void* host, size_t bytes, sb_buffer** out_buffer);
/* Allocates an uninitialised device buffer. */
SB_API sb_status sb_buffer_alloc(sb_session* session, const int64_t* shape, size_t rank, uint32_t elem_type,
                                 sb_buffer** out_buffer);
/* Asynchronous host -> device copy into an existing buffer (pinned host
 * memory makes it truly asynchronous). */
SB_API sb_status sb_buffer_h2d(sb_buffer* buffer, const void* host, size_t bytes);
/* Device -> host copy; waits at most timeout_ns (< 0 = no limit). */
SB_API sb_status sb_buffer_d2h(sb_buffer* buffer, void* host, size_t bytes, int64_t timeout_ns);
SB_API void sb_buffer_retain(sb_buffer* buffer);
SB_API void sb_buffer_release(sb_buffer* buffer);
/* Releases buffers[0 .. n) (null entries skipped) in one call: for a host
 * language whose foreign calls are costly, the outputs of a call it does not
 * keep. No counterpart in the reference (its values are dropped by Rust). */
SB_API void sb_buffer_release_many(sb_buffer* const* buffers, size_t n);
SB_API size_t sb_buffer_rank(const sb_buffer* buffer);
SB_API int64_t sb_buffer_dim(const sb_buffer* buffer, size_t axis);
SB_API uint32_t sb_buffer_elem_type(const sb_buffer* buffer);
SB_API size_t sb_buffer_byte_length(const sb_buffer* buffer);
SB_API void* sb_buffer_device_ptr(const sb_buffer* buffer);

/* ---- modules (replaces iree-compile + load_vmfb, jit/vag.rs:660-726,
 *      iree_session.rs:307-340) ---- */
/* Parses a StableHLO module as Sheaf's emitter prints it
 * (lowering/stablehlo/emit.rs:240-257) and maps it onto the kernel library.
 * An op the library cannot execute yields UNIMPLEMENTED, which the caller
 * treats like a failed compile (jit/compile.rs:119-125). The module is
 * registered in the session under its `module @<name>`. */
SB_API sb_status sb_module_load_stablehlo(sb_session* session, const char* mlir_text, size_t length,
                                          const char** out_module_name);
/* Parses and plans a StableHLO module without a device (the checks
 * sb_module_load_stablehlo makes before touching the GPU) and writes a short
 * summary (ops per function, arena size, recognised model) into `buf`.
 * UNIMPLEMENTED for ops outside the library's surface. */
SB_API sb_status sb_stablehlo_validate(const char* mlir_text, size_t length, char* buf, size_t capacity);

/* Writes a one-line-per-function description of how a loaded module executes
 * (fused nanoGPT plan, verified or not, or the generic op-by-op executor) into
 * `buf` (NUL-terminated, truncated to `capacity`). No reference counterpart:
 * IREE's equivalent is `--jit-profile` / the dispatch trace. */
SB_API sb_status sb_module_describe(sb_session* session, const char* module_name, char* buf, size_t capacity);

/* Registers the fused nanoGPT value_and_grad module (the graph of
 * examples/nanogpt/model.shf + cross-entropy) for a configuration without
 * going through text. Function "value_and_grad": inputs are the 4*...-leaf
 * parameter pytree in sorted-key order, then x ids [batch, seq] and y ids
 * [batch, seq] (f32); outputs are loss then one gradient per leaf. */
typedef struct sb_gpt_config {
  int32_t n_layer, n_head, n_embd, block_size, vocab_size, batch, seq;
  uint32_t elem_type; /* SB_ELEM_BF16 or SB_ELEM_F32 */
} sb_gpt_config;
SB_API sb_status sb_module_create_gpt_vag(sb_session* session, const char* module_name, const sb_gpt_config* config);

/* Registers the fused nanoGPT train-step module: the value_and_grad graph
 * followed by clip-by-global-norm(g, max_norm) and adamw-step(params, g, m, v,
 * t, lr, b1, b2, eps, weight_decay) (examples/nanogpt/train.shf:26-33,
 * lib/optim.shf:19-32,42-51), executed as one CUDA graph. train.shf's
 * constants are b1 0.9, b2 0.95, eps 1e-8, weight_decay 0.1, max_norm 1.0.
 * Function "train_step": inputs are the state pytree in sorted-key order --
 * loss [] (ignored), the m leaves, the parameter leaves, t [] f32, the v
 * leaves -- then x ids, y ids [batch, seq] (f32) and lr [] f32; m and v have
 * the parameters' element type. Outputs are the updated state in the same
 * order: loss, m', params', t + 1, v'. Function "value_and_grad" is also
 * available, as for sb_module_create_gpt_vag. */
typedef struct sb_adamw_config {
  float b1, b2, eps, weight_decay, max_norm; /* max_norm <= 0: no clipping */
} sb_adamw_config;
SB_API sb_status sb_module_create_gpt_train(sb_session* session, const char* module_name,
                                            const sb_gpt_config* config, const sb_adamw_config* adamw);

/* Registers the nanoGPT sampling module: generate-token of
 * examples/nanogpt/model.shf:116-125 repeated n_new times with the window
 * update of examples/nanogpt/sample.shf:28-45 (slide-window, key threading).
 * Each token runs the full-window forward (batch x block_size), takes the last
 * position's logits / temperature, top_k(min(top_k, vocab)), softmax,
 * random-split(key) and choice (sheaf/src/lowering/stablehlo/random_ops.rs:
 * 164-180), then appends the token and drops the oldest id. Sequence b uses
 * row b of ids and keys; with batch 1 this is the reference's generate.
 * config->seq must equal config->block_size and vocab_size must be <= 4096.
 * Function "generate": inputs are the parameter leaves in sorted-key order,
 * ids [batch, block_size] f32 and keys [batch, 4] f32 (four 16-bit limbs per
 * key, sheaf/src/core/prng.rs:29-40). Outputs: tokens [batch, n_new], the
 * final ids, the final keys and the last-position logits of every step
 * [n_new, batch, vocab] (all f32). */
typedef struct sb_sampler_config {
  int32_t n_new, top_k;
  float temperature;
} sb_sampler_config;
SB_API sb_status sb_module_create_gpt_sampler(sb_session* session, const char* module_name,
                                              const sb_gpt_config* config, const sb_sampler_config* sampler);

/* ---- invocation (replaces iree_runtime_session_call_by_name,
 *      iree_session.rs:576-583) ----
 * `qualified_name` is "<module>.<function>" (iree_dispatch.rs:95-104,172).
 * Inputs are borrowed for the call. On success `*out_count` outputs are
 * written to `outputs` (capacity `out_capacity`), each a new reference owned
 * by the caller. */
SB_API sb_status sb_call(sb_session* session, const char* qualified_name, sb_buffer* const* inputs, size_t in_count,
                         sb_buffer** outputs, size_t out_capacity, size_t* out_count);

/* ---- checkpoints: safetensors straight from / to device buffers
 *      (replaces io "save" / io "load" of .safetensors,
 *      sheaf/src/interpreter/builtins/safetensors.rs:13-81,200-331) ----
 * sb_safetensors_save writes the buffers under their keys exactly as the
 * reference's save_safetensors lays a file out (keys sorted, compact header
 * padded to an 8-byte boundary, raw little-endian data); the element type of
 * each buffer is its file dtype (F32, BF16, F16, I32). The file is written
 * under "<path>.tmp" and renamed into place. */
SB_API sb_status sb_safetensors_save(sb_session* session, const char* path, const char* const* keys,
                                     sb_buffer* const* buffers, size_t count);
/* Opens a safetensors file and parses its header (no device work). Entries
 * are listed in key order; "__metadata__" is skipped. */
typedef struct sb_safetensors_file_s sb_safetensors_file;
SB_API sb_status sb_safetensors_open(const char* path, sb_safetensors_file** out);
SB_API size_t sb_safetensors_count(const sb_safetensors_file* file);
SB_API const char* sb_safetensors_key(const sb_safetensors_file* file, size_t index);
/* Element type the entry loads as (F32/F64 -> SB_ELEM_F32, BF16, F16, and
 * I32/I64/U8/BOOL -> SB_ELEM_I32, following decode_raw) and its shape. */
SB_API sb_status sb_safetensors_info(const sb_safetensors_file* file, size_t index, uint32_t* elem_type,
                                     int64_t* shape, size_t shape_capacity, size_t* rank);
/* Reads entry `index` into a new device buffer (a reference owned by the
 * caller); the copy is complete when this returns. */
SB_API sb_status sb_safetensors_read(sb_session* session, const sb_safetensors_file* file, size_t index,
                                     sb_buffer** out);
SB_API void sb_safetensors_close(sb_safetensors_file* file);

#ifdef __cplusplus
}
#endif

#endif /* SHEAF_B200_H_ */
