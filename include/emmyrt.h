/*
 * emmyrt.h -- C ABI of libemmyrt.so, the B200 launcher for Emmy Kernel IR.
 *
 * The reference (ColonelToad/emmy-ptx) has no native library: its compiled
 * PTX goes over HTTP to a remote runner that assembles it (POST /compile,
 * docs/API.md:12-25) and launches it with the launch contract of meta.json
 * (POST /run, docs/API.md:26-38), driven by submit.py:84-159.  This library
 * is the local replacement for that runner on one B200: every entry point
 * below names the runner step (or submit.py step) it replaces.
 *
 * Conventions
 *   - Every function returns an int status: 0 = ok; a positive value is a
 *     CUresult / ncclResult_t code of the failing call; a negative value is
 *     one of the EMMY_E* codes.  emmy_last_error() gives a one-line message
 *     (thread-local), like the runner's "stderr" field.
 *   - The CUDA driver and NCCL are loaded with dlopen on first use, so the
 *     library itself loads (and reports a clean error) on machines without a
 *     GPU driver.
 *   - Device buffers are plain 64-bit device addresses (emmy_dptr) owned by
 *     the caller.  One context per device, used from one host thread; one
 *     process per GPU for multi-GPU work.
 */
#ifndef EMMYRT_H
#define EMMYRT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct emmy_ctx emmy_ctx;
typedef struct emmy_mod emmy_mod;
typedef struct emmy_comm emmy_comm;
typedef uint64_t emmy_dptr;
typedef void *emmy_stream; /* a CUstream; NULL is the legacy default stream */
typedef void *emmy_event;  /* a CUevent */

enum {
  EMMY_OK = 0,
  EMMY_ENODRIVER = -1,  /* libcuda.so.1 could not be loaded */
  EMMY_ENONCCL = -2,    /* libnccl.so.2 could not be loaded */
  EMMY_EINVAL = -3,     /* bad argument */
  EMMY_ENOENTRY = -4,   /* entry point not in module (runner stage "lookup") */
  EMMY_EKERNEL = -5,    /* a kernel reported an error in its error word */
  EMMY_ESYMBOL = -6,    /* module global not found */
  EMMY_ECUDART = -7     /* a CUDA runtime call failed (emmy_sum_f32_noalloc) */
};

/* Library identity and the last error message of the calling thread. */
const char *emmy_version(void);
const char *emmy_last_error(void);

/* ---- devices and contexts (replaces GET /health, docs/API.md:6-10) ---- */
int emmy_device_count(int *count);
/* Retain the primary context of `device` and make it current. */
int emmy_ctx_create(int device, emmy_ctx **out);
int emmy_ctx_destroy(emmy_ctx *ctx);
int emmy_ctx_make_current(emmy_ctx *ctx);
int emmy_ctx_synchronize(emmy_ctx *ctx);
/* name: at least 128 bytes. */
int emmy_device_info(emmy_ctx *ctx, int *sm_count, int *cc_major, int *cc_minor,
                     size_t *total_mem, char *name, int name_len);

/* ---- modules (replaces POST /compile, docs/API.md:12-25) ---- */
/* JIT-load PTX text.  On failure `log` (if given) receives the assembler's
 * error log, like the runner's "stderr" field for stage "ptxas". */
int emmy_module_load(emmy_ctx *ctx, const char *ptx, emmy_mod **out, char *log,
                     size_t log_len);
int emmy_module_unload(emmy_mod *mod);
/* Device address and size of a module-scope .global / .const variable. */
int emmy_module_global(emmy_mod *mod, const char *sym, emmy_dptr *ptr, size_t *bytes);
/* Per-entry facts (runner's "registers" field, docs/API.md:22-24). */
int emmy_func_info(emmy_mod *mod, const char *entry, int *regs, int *static_smem,
                   int *max_threads, int *local_bytes);

/* ---- launches (replaces POST /run, docs/API.md:26-38) ---- */
/* `args` is the cuLaunchKernel parameter array: one pointer per kernel
 * parameter, in the entry's parameter order (meta.json arg_order).
 * Dynamic shared memory above 48 KiB is opted into automatically. */
int emmy_launch(emmy_mod *mod, const char *entry, const uint32_t grid[3],
                const uint32_t block[3], uint32_t smem_bytes, void **args, emmy_stream stream);
/* Same, for the common case where every parameter is a .u64 buffer address. */
int emmy_launch_ptrs(emmy_mod *mod, const char *entry, const uint32_t grid[3],
                     const uint32_t block[3], uint32_t smem_bytes, const emmy_dptr *ptrs,
                     int nptrs, emmy_stream stream);
/* emmy_launch with flags.  EMMY_LAUNCH_OVERLAP_PREV: the grid may start
 * while the previous kernel in `stream` finishes (programmatic dependent
 * launch).  Only for kernels whose plan declares "overlap" (they wait for
 * the previous kernel before their first write) and only when none of
 * their inputs is written by that previous kernel -- the caller's promise.
 * Replaces the same runner step as emmy_launch; the overlap is new. */
enum { EMMY_LAUNCH_OVERLAP_PREV = 1 };
int emmy_launch_ex(emmy_mod *mod, const char *entry, const uint32_t grid[3],
                   const uint32_t block[3], uint32_t smem_bytes, void **args, emmy_stream stream,
                   uint32_t flags);

/* ---- TMA tensor maps kept in module globals ---- */
/* A kernel parameter list is fixed by meta.json arg_order, so tensor maps
 * live in 64-byte-aligned 128-byte module globals that the launcher fills
 * before the launch (stream-ordered). */
typedef struct {
  emmy_dptr base;       /* global address of element (0,...,0), 16-byte aligned */
  uint32_t rank;        /* 1..5 */
  uint32_t dtype;       /* EMMY_TMAP_F32 / BF16 / F16 / U8 */
  uint64_t dims[5];     /* extents, innermost first */
  uint64_t strides[4];  /* byte strides of dims 1..rank-1 (multiples of 16) */
  uint32_t box[5];      /* box extents, innermost first */
  uint32_t swizzle;     /* 0, 32, 64 or 128 (bytes) */
  uint32_t l2_promote;  /* 0 none, 64, 128, 256 (bytes) */
} emmy_tmap_desc;

enum { EMMY_TMAP_F32 = 0, EMMY_TMAP_BF16 = 1, EMMY_TMAP_F16 = 2, EMMY_TMAP_U8 = 3 };

/* Encode `desc` into the 128-byte CUtensorMap at `out` (host memory). */
int emmy_tmap_encode(const emmy_tmap_desc *desc, void *out128);
/* Encode and copy into module global `sym` on `stream`. */
int emmy_tmap_fill(emmy_mod *mod, const char *sym, const emmy_tmap_desc *desc,
                   emmy_stream stream);

/* ---- memory (the runner's argument forms, docs/API.md:40-50) ---- */
int emmy_mem_alloc(emmy_ctx *ctx, size_t bytes, emmy_dptr *out);
int emmy_mem_free(emmy_ctx *ctx, emmy_dptr ptr);
int emmy_host_alloc(emmy_ctx *ctx, size_t bytes, void **out); /* pinned */
int emmy_host_free(emmy_ctx *ctx, void *ptr);
int emmy_memcpy_htod(emmy_dptr dst, const void *src, size_t bytes, emmy_stream stream);
int emmy_memcpy_dtoh(void *dst, emmy_dptr src, size_t bytes, emmy_stream stream);
int emmy_memcpy_dtod(emmy_dptr dst, emmy_dptr src, size_t bytes, emmy_stream stream);
/* "zero_outputs": buffers re-zeroed before every launch (docs/API.md:31). */
/* Peer inboxes for the fused cross-GPU reduction (no counterpart in the
 * reference, which has no multi-GPU path): export a device allocation as a
 * 64-byte IPC handle, open a peer process's handle (peer access enabled
 * lazily; the returned pointer addresses the peer GPU's memory over
 * NVLink), close it. */
int emmy_ipc_handle(emmy_ctx *ctx, emmy_dptr ptr, void *out64);
int emmy_ipc_open(emmy_ctx *ctx, const void *handle64, emmy_dptr *out);
int emmy_ipc_close(emmy_ctx *ctx, emmy_dptr ptr);

int emmy_memset_d32(emmy_dptr dst, uint32_t value, size_t count, emmy_stream stream);

/* ---- streams and events (the runner's median_us timing) ---- */
int emmy_stream_create(emmy_ctx *ctx, emmy_stream *out);
int emmy_stream_destroy(emmy_stream stream);
int emmy_stream_sync(emmy_stream stream);
int emmy_event_create(emmy_ctx *ctx, emmy_event *out);
int emmy_event_destroy(emmy_event ev);
int emmy_event_record(emmy_event ev, emmy_stream stream);
int emmy_event_elapsed(emmy_event start, emmy_event end, float *ms);
/* Make `stream` wait for `ev` (overlap of NCCL on a second stream with the
 * next kernels; no counterpart in the single-stream reference runner). */
int emmy_stream_wait_event(emmy_stream stream, emmy_event ev);

/* ---- kernel error word ---- */
/* Kernels that can fail (bounded waits that expire, index checks in the
 * checked build) write a nonzero code into the module global `emmy_err`
 * instead of trapping.  Reads it after synchronising `stream`, optionally
 * clears it.  Returns EMMY_ESYMBOL if the module has no error word. */
int emmy_error_word(emmy_mod *mod, uint32_t *value, int clear, emmy_stream stream);

/* ---- NCCL over NVLink (no counterpart in the reference, which is
 *      single-GPU; used for full reductions sharded across GPUs) ---- */
int emmy_nccl_unique_id(void *out128);
int emmy_nccl_init(emmy_ctx *ctx, int nranks, int rank, const void *id128, emmy_comm **out);
int emmy_allreduce_sum_f32(emmy_comm *comm, emmy_dptr buf, size_t count, emmy_stream stream);
int emmy_nccl_async_error(emmy_comm *comm, int *nccl_result);
int emmy_nccl_abort(emmy_comm *comm);
int emmy_nccl_destroy(emmy_comm *comm);

/* ---- full f32 sum without any allocation ----
 * No counterpart in the reference.  For callers that cannot call cudaMalloc
 * where they need the reduction: plugin hosts whose enqueue callback must
 * not allocate because the host framework owns all device memory, and
 * latency-critical loops where cudaMalloc's implicit device-wide
 * synchronisation would stall other streams.  *out = sum of the n f32 at x
 * (x 16-byte aligned, out 4-byte aligned, 1 <= n <= 2^31 - 1, else
 * EMMY_EINVAL), on `stream` (the CUDA runtime's current device, in the
 * context current on the calling thread).  It allocates nothing: its
 * scratch is a 4.25 KiB file-scope device array (1024 per-CTA partials + a
 * ticket) held by every GPU that loads this library until exit.  The first
 * call in each context resolves that array's address (cudaGetSymbolAddress)
 * -- make it before any stream capture; the resolved address is not
 * refreshed after cudaDeviceReset, so do not call this after resetting the
 * device.  All calls on a device share the array and each clears the ticket
 * first; calls that overlap on the GPU race and must be serialised by the
 * caller.  A failing CUDA runtime call returns EMMY_ECUDART (its message in
 * emmy_last_error()), never a raw cudaError_t. */
int emmy_sum_f32_noalloc(emmy_dptr x, size_t n, emmy_dptr out, emmy_stream stream);

#ifdef __cplusplus
}
#endif
#endif /* EMMYRT_H */
