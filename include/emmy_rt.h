/*
 * emmy_rt.h -- C ABI of the B200 runtime that loads and launches the PTX
 * emitted by compile.py.
 *
 * The reference has no native runtime: its harness posts PTX to a remote
 * runner over HTTP (reference submit.py:99-137, docs/API.md:14-56). This
 * library is that runner's local, in-process replacement on B200, and it is
 * the boundary a host program binds (ctypes, cgo, JNI ...). Every entry
 * point takes plain pointers and sizes; none takes a PyTorch type.
 *
 * The CUDA driver (libcuda.so.1) is opened lazily with dlopen, so the
 * library loads on machines without a GPU; every call then fails with
 * EMMY_RT_ENODRIVER.
 *
 * Return values: 0 on success, a negative EMMY_RT_* code on failure. The
 * message of the last failure on the calling thread is available from
 * emmy_rt_last_error().
 */
#ifndef EMMY_RT_H
#define EMMY_RT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EMMY_RT_ABI_VERSION 1

#define EMMY_RT_OK 0
#define EMMY_RT_ENODRIVER (-1)   /* libcuda.so.1 missing or incomplete          */
#define EMMY_RT_ECUDA (-2)       /* a driver call failed (message has details)  */
#define EMMY_RT_EINVAL (-3)      /* bad argument                                 */
#define EMMY_RT_ENOTFOUND (-4)   /* entry point or symbol not in the module      */
#define EMMY_RT_ETIMEOUT (-5)    /* bounded wait expired                         */
#define EMMY_RT_EKERNEL (-6)     /* the kernel raised its module error word      */

typedef struct emmy_module emmy_module;   /* one loaded PTX module (one entry)  */

/* Run-call argument (docs/API.md:41-56 "Argument forms"). */
typedef struct emmy_arg {
  void *host;          /* host buffer: input data, or output destination        */
  uint64_t bytes;      /* buffer size in bytes                                   */
  int32_t is_output;   /* 1: allocated zeroed and copied back after the run       */
  int32_t zero_each;   /* 1: re-zeroed before EVERY launch ("zero_outputs")      */
} emmy_arg;

/* Timing summary of emmy_rt_run: medians over the timed iterations. */
typedef struct emmy_run_stats {
  float kernel_us_median;   /* launch only (CUDA events around cuLaunchKernel)  */
  float e2e_us_median;      /* H2D inputs + zeroing + launch + D2H outputs      */
  uint64_t h2d_bytes;       /* bytes copied host->device per iteration          */
  uint64_t d2h_bytes;       /* bytes copied device->host per iteration          */
  int32_t iters;
} emmy_run_stats;

/* ABI version this library was built with (EMMY_RT_ABI_VERSION). */
int emmy_rt_abi_version(void);

/* Message of the last failure on this thread ("" if none). */
const char *emmy_rt_last_error(void);

/* cuInit, select `device`, retain its primary context and make it current
 * on the calling thread. The primary context is the one the CUDA runtime
 * (and PyTorch) uses, so device pointers are shared both ways. */
int emmy_rt_init(int device);

/* Device facts for launch sizing: SM count, compute capability, L2 bytes,
 * max dynamic shared memory per block. Any out pointer may be NULL. */
int emmy_rt_device_info(int device, int *sm_count, int *cc_major, int *cc_minor,
                        int *l2_bytes, int *max_smem_optin, char *name, size_t name_size);

/* JIT-load PTX text (NUL-terminated) for the current device and resolve its
 * entry `entry`. Replaces POST /compile + entry lookup (docs/API.md:14-24,
 * reference submit.py:99-110). On failure the JIT log is copied to `log`. */
int emmy_rt_module_load(const char *ptx, const char *entry, emmy_module **out, char *log,
                        size_t log_size);
int emmy_rt_module_unload(emmy_module *m);

/* Registers per thread, static shared bytes and max threads per block of
 * the entry (the runner's "registers" field, docs/API.md:18-24). */
int emmy_rt_module_attrs(emmy_module *m, int *num_regs, int *static_smem, int *max_threads);

/* Read (and with clear=1 reset) the module-scope word `emmy_error` that
 * bounded device-side waits set instead of hanging. 0 if the module has no
 * such word. */
int emmy_rt_module_error_word(emmy_module *m, uint32_t *value, int clear);

/* Device address and size of a module-scope .global symbol. */
int emmy_rt_module_global(emmy_module *m, const char *name, uint64_t *dptr, uint64_t *bytes);

/* Tensor maps (no counterpart in the reference: its PTX ABI passes pointers only). A kernel
 * that can load tiles with TMA (the attention template) declares a table `emmy_tmap_desc` of
 * the maps it wants: per map the parameter index, rank, dims, byte strides, box, swizzle,
 * data type and L2 promotion. Before a launch whose pointers differ from the ones the maps
 * were last written for, every launch function of this library encodes them
 * (cuTensorMapEncodeTiled) and copies them with their keys (the pointers) into the module's
 * globals on the launch stream, after waiting for the module's earlier launches. The kernel
 * uses TMA only when every key equals its own parameter and otherwise stages tiles through
 * registers, so results never depend on the maps; a runner that does not write them (the
 * reference's) gets the register path. Launches under stream capture never write maps, and
 * after one the module's maps are frozen. Pointers TMA cannot take (not 16-byte aligned)
 * leave the maps as they are.
 * enable: 1 = write maps (the default), 0 = stop writing them and clear the keys (later
 * launches take the register path; waits for the module's launches and the context), -1 =
 * query only. nmaps: maps the module declares (0: none, or a driver without
 * cuTensorMapEncodeTiled); uploads: map writes so far. */
int emmy_rt_module_tensor_maps(emmy_module *m, int enable, int *nmaps, uint64_t *uploads);

/* Launch with device-pointer arguments in arg_order (each a .u64 param).
 * Dynamic shared memory above 48 KiB is enabled on the function first, as
 * the runner does for meta.json smem_bytes (reference PROVENANCE.md). */
int emmy_rt_launch(emmy_module *m, const uint32_t grid[3], const uint32_t block[3],
                   uint32_t smem_bytes, const uint64_t *args, int nargs, uint64_t stream);

/* emmy_rt_launch with launch flags. EMMY_RT_LAUNCH_OVERLAP launches with
 * programmatic stream serialization (cuLaunchKernelEx): the grid may start
 * while the previous kernel on the stream finishes, as soon as every CTA of
 * that kernel has executed griddepcontrol.launch_dependents. The full sum and
 * mean kernels this compiler emits execute it once a thread has streamed 7/8
 * of its input (the next kernel then reads lines this one read more than an
 * L2's worth of bytes earlier, for inputs larger than L2), and run
 * griddepcontrol.wait before any global write: only for back-to-back launches
 * whose inputs the previous kernel does not write. The pointwise and row
 * kernels execute both at entry, before any global access, so only the launch
 * latency overlaps and a chain of launches (one's output the next one's
 * input) keeps its order. Under a plain launch both instructions do nothing.
 * Not part of the reference runner's interface (an addition of this
 * library). */
#define EMMY_RT_LAUNCH_OVERLAP 1u
int emmy_rt_launch_ex(emmy_module *m, const uint32_t grid[3], const uint32_t block[3],
                      uint32_t smem_bytes, const uint64_t *args, int nargs, uint64_t stream,
                      uint32_t flags);

/* Wait for `stream` (0 = legacy default stream) with a wall-clock bound. */
int emmy_rt_sync(uint64_t stream, int timeout_ms);

/* Time `iters` launches after `warmup` untimed ones, each bracketed by CUDA
 * events on `stream`. If flush_bytes > 0 the buffer at flush_ptr is
 * rewritten (cuMemsetD32Async) before every launch so each one starts with a
 * cold L2. Per-launch milliseconds go to ms_out[iters]. */
int emmy_rt_time(emmy_module *m, const uint32_t grid[3], const uint32_t block[3],
                 uint32_t smem_bytes, const uint64_t *args, int nargs, uint64_t stream,
                 int warmup, int iters, uint64_t flush_ptr, uint64_t flush_bytes, float *ms_out);

/* Runner-equivalent run with HOST buffers (POST /run, docs/API.md:25-56;
 * reference submit.py:112-137): allocate device buffers, then per
 * iteration copy inputs host->device, zero outputs ("zero_outputs" args
 * before every launch, all outputs before the first), launch, copy outputs
 * back. Timing covers the copies (e2e) and the launch alone (kernel). */
int emmy_rt_run(emmy_module *m, const uint32_t grid[3], const uint32_t block[3],
                uint32_t smem_bytes, emmy_arg *args, int nargs, int warmup, int iters,
                emmy_run_stats *stats);

/* Device memory helpers for hosts without their own allocator. */
int emmy_rt_mem_alloc(uint64_t bytes, uint64_t *dptr);
int emmy_rt_mem_free(uint64_t dptr);
int emmy_rt_memcpy_htod(uint64_t dst, const void *src, uint64_t bytes);
int emmy_rt_memcpy_dtoh(void *dst, uint64_t src, uint64_t bytes);
int emmy_rt_memset_zero(uint64_t dptr, uint64_t bytes);
/* Page-locked host memory (fast H2D/D2H for emmy_rt_run). */
int emmy_rt_host_alloc(uint64_t bytes, void **ptr);
int emmy_rt_host_free(void *ptr);

/* ---- allocation-free f32 sum --------------------------------------------
 * No counterpart in the reference: it adds nothing to the PTX contract and
 * exists for hosts that may not allocate device memory while they call this
 * library (for example a service whose pool has already reserved the GPU's
 * memory, or a timing loop in which a cudaFree would synchronise the device).
 *
 * out[0] = sum of the n floats at x, with `grid` CTAs of 256 threads on
 * `stream` (0 = legacy default stream) of the current device. The scratch
 * for the cross-CTA finish is a fixed array inside this library (16,640 bytes
 * per device, held until the process exits), so at most
 * EMMY_RT_NOALLOC_MAX_CTAS CTAs are accepted; larger grids return
 * EMMY_RT_EINVAL with a message. The call allocates nothing. All calls on a
 * device share that array: calls that overlap on the GPU race and must be
 * serialised. x and out must be 4-byte aligned, else EMMY_RT_EINVAL before
 * any launch. The first call on a device looks up the array's address
 * (cudaGetSymbolAddress); under CUDA's lazy module loading (the default since
 * CUDA 12.2) that first call also loads this code and its array onto the
 * device, so make it before the host's pool reserves the device's memory and
 * before any stream capture. Later calls outside capture look the address up
 * again (a reset context is picked up); calls on a capturing stream reuse the
 * last address found. */
#define EMMY_RT_NOALLOC_MAX_CTAS 4096
int emmy_rt_sum_f32_noalloc(uint64_t x, uint64_t n, uint64_t out, uint32_t grid,
                            uint64_t stream);

/* ---- cross-GPU fold over peer memory ------------------------------------
 * No counterpart in the reference (which runs one GPU per kernel): a sharded
 * full reduction leaves each rank (one process per GPU) with partial scalars
 * whose sum over ranks is the result. emmy_rt_fold_f32 adds `nvals` (1..4)
 * floats at `vals` over all `world` ranks into out[0..nvals) on every rank,
 * in rank order (every rank gets the same bits), with one 32-thread CTA on
 * `stream`. `boxes` is a device array of `world` pointers: boxes[r] is rank
 * r's mailbox (EMMY_RT_FOLD_BOX_BYTES(world) bytes, 16-byte aligned, zeroed
 * before the first call, allocated with emmy_rt_mem_alloc), mapped into this process with
 * emmy_rt_ipc_open for r != rank. The kernel stores this rank's values and a
 * flag into every mailbox (NVLink peer stores, system-scope release) and
 * waits for every rank's flag in its own. `epoch` counts the calls from 1;
 * every rank makes the same sequence of calls. A wait is bounded (about one
 * second): a rank that never arrives sets bit 0 of the u32 at `err` and the
 * kernel returns without writing out; while that word is nonzero, later calls
 * return at once without writing out (the host clears it). With EMMY_RT_LAUNCH_OVERLAP in `flags`
 * the fold lets the next kernel on the stream start at once (it executes
 * griddepcontrol.launch_dependents first) and reads `vals` only after the
 * previous kernel completed (griddepcontrol.wait). */
#define EMMY_RT_FOLD_BOX_BYTES(world) (64u * (uint32_t)(world))
int emmy_rt_fold_f32(uint64_t vals, uint32_t nvals, uint64_t boxes, uint32_t rank,
                     uint32_t world, uint32_t epoch, uint64_t out, uint64_t err,
                     uint64_t stream, uint32_t flags);
/* CUDA IPC for the mailboxes: the 64-byte handle of an allocation made with
 * emmy_rt_mem_alloc, its mapping in another process on the same node (peer
 * access enabled), and the unmapping. A process cannot open its own handle. */
#define EMMY_RT_IPC_HANDLE_BYTES 64
int emmy_rt_ipc_handle(uint64_t dptr, void *handle);
int emmy_rt_ipc_open(const void *handle, uint64_t *dptr);
int emmy_rt_ipc_close(uint64_t dptr);

#ifdef __cplusplus
}
#endif

#endif /* EMMY_RT_H */
