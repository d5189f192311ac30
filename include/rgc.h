/* rgc — the CUDA execution device for rg's compiled step plans, as a C ABI.
 *
 * This is the boundary a `src/cuda.rs` device module in rg would bind, beside
 * `src/metal.rs` / `src/metal_stub.rs` behind the `lib.rs:4-8` device switch. Each entry point
 * replaces one piece of the Metal device's contract (reference paths relative to the rg repo):
 *
 *   rgc_available               metal.rs:58-60        `available()`
 *   rgc_program_create          metal.rs:381-383      `MetalProgram::new(&Plan)` (kernel build, buffer limits)
 *   rgc_program_destroy         metal.rs:362-379      drop of `MetalProgram`
 *   rgc_program_allocated_bytes metal.rs:386-388      `allocated_bytes()`
 *   rgc_program_inject_failure  metal.rs:527-529      `inject_failure_for_test()`
 *   rgc_exec_acquire            metal.rs:506-523      `MetalProgram::exec(&Plan)` (pooled frames, constants resident)
 *   rgc_exec_release            metal.rs:565-571      drop of `MetalExec` (frame returns to the pool)
 *   rgc_exec_load               plan.rs:31            `Exec::load`
 *   rgc_exec_step               plan.rs:32            `Exec::step`
 *   rgc_exec_step_at            (one plan step; the instrumented validation runs of validate.rs:541-565)
 *   rgc_exec_swap               plan.rs:33            `Exec::swap`
 *   rgc_exec_prefix             plan.rs:34            `Exec::prefix`
 *   rgc_exec_write_prefix       plan.rs:35            `Exec::write_prefix`
 *   rgc_exec_scalar             plan.rs:36            `Exec::scalar`
 *   rgc_exec_failure            plan.rs:38-40         `Exec::failure`
 *   rgc_exec_run                validate.rs:290-363   `run_loop`, kept on the device (no host sync per step)
 *   rgc_exec_step_checked       validate.rs:132-230   the non-finite observer's per-step scan, on the device
 *   rgc_exec_save_slots/_load_slots checkpoint.py:37-105 safetensors checkpoints, device <-> file
 *   rgc_exec_step_timed         metal.rs:692-700      `step_timed`
 *   rgc_exec_breakdown_json     metal.rs:701-712      `breakdown`
 *   rgc_dist_*                  (new) data-parallel communicator for the gradient all-reduce step
 *
 * Plans cross the ABI as one byte string (the "plan blob"): magic "RGPL", u32 version 1, then
 * the plan (slots, pinned flags, constants, input and output slots, steps with nested
 * control-flow body plans), little-endian, as written by rg's plan serialiser. All functions
 * return 0 on success and a negative code on failure; `rgc_last_error` then describes it.
 * No C++ exception crosses this boundary. Host pointers are plain host memory.
 */
#ifndef RGC_H
#define RGC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RGC_OK 0
#define RGC_ERR_INVALID (-1)     /* malformed plan blob or argument */
#define RGC_ERR_CUDA (-2)        /* CUDA runtime or NVRTC error */
#define RGC_ERR_UNAVAILABLE (-3) /* no usable sm_100 device */
#define RGC_ERR_DEVICE (-4)      /* the device reported a failure (sticky for this exec) */

typedef struct rgc_program rgc_program;
typedef struct rgc_exec rgc_exec;

/* 1 when an sm_100 CUDA device is present and usable, else 0. Safe without a GPU. */
int rgc_available(void);
/* Message for the last failing call on this thread (empty string if none). */
const char* rgc_last_error(void);

/* Lowers a plan onto kernels for the current CUDA device; `device` < 0 means the current one. */
int rgc_program_create(const uint8_t* plan, size_t len, int device, rgc_program** out);
void rgc_program_destroy(rgc_program* p);
size_t rgc_program_allocated_bytes(const rgc_program* p);
/* The next step of any exec of this program fails, as a device failure would. */
void rgc_program_inject_failure(rgc_program* p);

/* A frame of device buffers with the constants loaded; frames are pooled per program. */
int rgc_exec_acquire(rgc_program* p, rgc_exec** out);
void rgc_exec_release(rgc_exec* e);
/* Copies `bytes` from host memory into input `input` (its first bytes). */
int rgc_exec_load(rgc_exec* e, size_t input, const void* host, size_t bytes);
int rgc_exec_step(rgc_exec* e);
int rgc_exec_step_at(rgc_exec* e, size_t step);
int rgc_exec_swap(rgc_exec* e, size_t slot_a, size_t slot_b);
/* Copies the first `bytes` of slot `slot` to host memory (synchronises). */
int rgc_exec_prefix(rgc_exec* e, size_t slot, void* host, size_t bytes);
int rgc_exec_write_prefix(rgc_exec* e, size_t slot, const void* host, size_t bytes);
int rgc_exec_scalar(rgc_exec* e, size_t slot, double* out);
/* 1 and the reason in `buf` if the exec has failed, else 0. */
int rgc_exec_failure(rgc_exec* e, char* buf, size_t cap);
/* Device pointer of a slot, for zero-copy interop (valid until the next swap or release). */
int rgc_exec_slot_pointer(rgc_exec* e, size_t slot, void** out);

/* The multi-step run (validate.rs:290-363) on the device.
 * state_inputs/state_outputs: n_state (input index, output index) pairs fed back each step.
 * `state` NULL: the state inputs already hold the state (left by an earlier run on this exec, or
 * written by rgc_exec_load / rgc_exec_load_slots), so nothing is uploaded.
 * data_inputs: n_data input indices loaded from `batches`, cycled one batch per step.
 * history_outputs: n_history scalar outputs recorded per step into `history` (row-major
 * [n_history][steps], doubles). State and batch tensors are host memory: state[k] has the bytes
 * of input state_inputs[k]; batches[b * n_data + d] is data input d of batch b.
 * On return, *steps_done steps completed; *nonfinite_step is the first step with a
 * non-finite history scalar or -1; the final state is in the state input slots (read it with
 * rgc_exec_prefix on those inputs' slots) and, if `outputs` is not NULL, outputs[k] receives
 * output k of the last completed step (`output_bytes[k]` bytes). *seconds is device time. */
typedef struct {
  const size_t* state_inputs;
  const size_t* state_outputs;
  size_t n_state;
  const size_t* data_inputs;
  size_t n_data;
  const size_t* history_outputs;
  size_t n_history;
} rgc_run_spec;

int rgc_exec_run(rgc_exec* e, const rgc_run_spec* spec, const void* const* state, const void* const* batches,
                 size_t n_batches, size_t steps, double* history, void* const* outputs, const size_t* output_bytes,
                 size_t* steps_done, int64_t* nonfinite_step, double* seconds);

/* One step with a check after every plan step, for validate's non-finite observer
 * (validate.rs:132-230) on large plans: flags[k] = 1 when plan step k produced a non-finite
 * value (every float output of the step, fused groups included), flags[n + k] = 1 when an index
 * read by step k (take, take_along) lay outside its axis; n = number of plan steps, the array
 * holds 2n entries. */
int rgc_exec_step_checked(rgc_exec* e, int32_t* flags, size_t n_flags);

/* Checkpoints straight between device slots and a file (checkpoint.py:37-105 writes and reads
 * the same safetensors layout from host tensors). Save writes `path` through a temporary file
 * renamed into place: the 8-byte little-endian header length, `header` (header_len bytes), then
 * sizes[k] bytes of slots[k] in order, streamed through pinned host memory. Load reads sizes[k]
 * bytes at file offsets[k] into slots[k]. */
int rgc_exec_save_slots(rgc_exec* e, const char* path, const char* header, size_t header_len, const size_t* slots, const size_t* sizes,
                        size_t n);
int rgc_exec_load_slots(rgc_exec* e, const char* path, const uint64_t* offsets, const size_t* slots, const size_t* sizes, size_t n);

/* Per-step device seconds, accumulated into seconds[n_steps] (metal.rs:692-700). */
int rgc_exec_step_timed(rgc_exec* e, double* seconds, size_t n_steps);
/* JSON object describing where a step's time goes; writes at most `cap` bytes. */
int rgc_exec_breakdown_json(rgc_exec* e, size_t repeats, char* buf, size_t cap);

/* Kernel launches issued since the program was created (all execs), for accounting. */
uint64_t rgc_program_launches(const rgc_program* p);

/* Sum of the `n` elements of the device array `src` (dtype 0 = float32, 1 = float64) into the
 * one-element device array `dst`, enqueued on `stream` (a cudaStream_t; NULL = the legacy default
 * stream). Same kernels and summation order as a plan's full-tensor Sum, so the result is
 * bit-identical to it. No counterpart in the reference: it exists for callers that may not
 * allocate device memory when they need the sum (an allocator's own callbacks or out-of-memory
 * handler, a host whose memory pool owns the whole device heap, a loop where cudaMalloc's
 * implicit synchronisation is not allowed). It allocates nothing: the partial sums go to a fixed
 * 256 KiB array in the library (held on every GPU that loads it until exit), which limits n to
 * 2^29 float32 or 2^28 float64 elements; larger n fails with RGC_ERR_INVALID before any launch.
 * The array needs no clearing between calls, but all calls on a device share it, so calls that
 * may overlap on the GPU race. The first call on a device does set-up (looks up the array's
 * address, loads the kernels): make it before beginning any stream capture. */
int rgc_sum_noalloc(const void* src, int64_t n, int dtype, void* dst, void* stream);

/* Data parallelism: one process per GPU; rank 0 creates the id, every rank joins. */
int rgc_dist_unique_id(uint8_t id[128]);
int rgc_dist_init(int rank, int world, const uint8_t id[128]);
int rgc_dist_finalize(void);

#ifdef __cplusplus
}
#endif

#endif /* RGC_H */
