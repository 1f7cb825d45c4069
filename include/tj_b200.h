/*
 * tj_b200.h — C ABI of the B200 execution runtime for tensorjit kernel plans.
 *
 * The runtime executes one compiled program: a straight-line list of kernels
 * (sm_100a cubins produced from the plan) whose arguments are resolved, per
 * call, to caller inputs, caller outputs, or offsets into a device arena that
 * the runtime owns.  It replaces the reference's GPU execution path:
 *
 *   - tensorjit/backends/cuda_driver.py:99-131  Module (cuModuleLoadData,
 *     cuLaunchKernel on the current stream)      -> tj_b200_program_create / tj_b200_run
 *   - tensorjit/backends/cuda_driver.py:134-168 Graph (stream capture, replay)
 *                                                -> tj_b200_set_graph + tj_b200_run
 *   - tensorjit/backends/cuda_backend.py:459-553 CudaProgram (arena, arg
 *     resolution node -> input/arena/output)     -> tj_argref + arena owned here
 *   - csrc/runtime.cpp:31-110 ArgKind INPUT/ARENA/OUTPUT and Program::run of
 *     the native runtime                          -> same argument-reference scheme
 *
 * All functions return TJ_OK (0) or a negative TJ_ERR_* code; the message of
 * the last failure on the calling thread is returned by tj_b200_last_error().
 * Handles and pointers are plain C types: device pointers are void*, streams
 * are CUstream values passed as void*.  The library loads libcuda lazily, so it
 * can be loaded (and its symbols listed) on a machine without a GPU.
 */
#ifndef TJ_B200_H
#define TJ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TJ_B200_ABI_VERSION 1

#if defined(__GNUC__)
#define TJ_API __attribute__((visibility("default")))
#else
#define TJ_API
#endif

enum {
  TJ_OK = 0,
  TJ_ERR_INVALID = -1,       /* bad argument, arity or range */
  TJ_ERR_CUDA = -2,          /* a CUDA driver call failed */
  TJ_ERR_NO_DRIVER = -3,     /* libcuda could not be loaded */
  TJ_ERR_DEVICE_STATUS = -4, /* a kernel reported a failed bounded wait or check */
  TJ_ERR_NOT_SUPPORTED = -5
};

/* Where a kernel argument lives (csrc/runtime.cpp:31 ArgKind, plus STATUS). */
enum {
  TJ_ARG_INPUT = 0,   /* value = index of the caller input            */
  TJ_ARG_ARENA = 1,   /* value = byte offset into the program's arena */
  TJ_ARG_OUTPUT = 2,  /* value = index of the caller output           */
  TJ_ARG_STATUS = 3   /* the program's device status words (int32[4]) */
};

typedef struct tj_argref {
  int32_t kind;
  int32_t reserved;
  int64_t value;
} tj_argref;

/* A TMA descriptor built at run time from one resolved argument. */
typedef struct tj_tmap {
  int32_t arg;            /* index (within the kernel's argrefs) of the base pointer */
  int32_t dtype;          /* CUtensorMapDataType */
  int32_t rank;           /* 1..5 */
  int32_t swizzle;        /* CUtensorMapSwizzle */
  uint64_t dims[5];       /* elements, innermost first */
  uint64_t strides[4];    /* bytes, for dims 1..rank-1 */
  uint32_t box[5];        /* elements, innermost first */
  uint32_t param_offset;  /* byte offset of the CUtensorMap in the parameter block */
  int32_t l2_promotion;   /* CUtensorMapL2promotion */
  int32_t reserved;
} tj_tmap;

/* One kernel launch.  The kernel takes ONE by-value parameter block of
 * param_bytes bytes: num_args device pointers at offsets 0, 8, 16, ...,
 * followed by the CUtensorMaps at their param_offset. */
typedef struct tj_launch {
  const char* symbol;     /* entry point name in module `module` */
  int32_t module;         /* index into the cubin list */
  uint32_t grid[3];       /* a zero extent skips the launch (empty tensors) */
  uint32_t block[3];
  uint32_t cluster[3];    /* 0 or 1 = no cluster; a cluster launch must be a persistent kernel
                             (work strided by gridDim): its grid is clamped at create time to the
                             number of clusters that can be resident at once */
  uint32_t smem_bytes;    /* dynamic shared memory */
  uint32_t param_bytes;
  int32_t first_arg, num_args;
  int32_t first_tmap, num_tmaps;
} tj_launch;

typedef struct tj_program_info {
  void* arena;               /* device address of the arena (NULL if 0 bytes) */
  uint64_t arena_bytes;
  int32_t num_kernels;
  int32_t num_inputs;
  int32_t num_outputs;
  int32_t graph_enabled;
  uint64_t calls;            /* tj_b200_run calls */
  uint64_t launches;         /* kernel launches issued directly (non-graph) */
  uint64_t graph_replays;    /* cuGraphLaunch calls */
  uint64_t graph_node_updates; /* kernel nodes re-pointed at new caller buffers */
  uint64_t graph_instantiations;
  double host_us_total;      /* host time spent inside tj_b200_run */
} tj_program_info;

/* Load `num_modules` sm_100a cubins and bind a program to device `device`.
 * Replaces cuda_backend.py:462-491 (CudaProgram.__init__: module load, arena). */
TJ_API int tj_b200_program_create(const void* const* cubins, const size_t* cubin_sizes, int32_t num_modules,
                           const tj_launch* launches, int32_t num_kernels,
                           const tj_argref* args, int32_t num_args_total,
                           const tj_tmap* tmaps, int32_t num_tmaps_total,
                           uint64_t arena_bytes, int32_t num_inputs, int32_t num_outputs,
                           int32_t device, void** out_program);

/* Run the whole program on `stream` (a CUstream; NULL = legacy default stream).
 * inputs[i] / outputs[j] are device pointers of contiguous buffers.
 * Replaces cuda_backend.py:516-540 (CudaProgram.__call__) and
 * csrc/runtime.cpp:88-110 (Program::run). */
TJ_API int tj_b200_run(void* program, const void* const* inputs, void* const* outputs, void* stream);

/* Whole-program CUDA graph on/off (default off).  With it on, the first run
 * builds and instantiates one graph of all kernels; later runs replay it and
 * re-point only the kernel nodes whose caller buffers changed, so inputs are
 * never copied into static buffers.  Replaces cuda_driver.py:134-168. */
TJ_API int tj_b200_set_graph(void* program, int32_t enable);

/* Run the program `iters` times without a graph, with a CUDA event recorded on
 * `stream` before every kernel; ms_per_kernel[k] (num_kernels floats) receives
 * the mean device time of kernel k.  Used for per-kernel rooflines. */
TJ_API int tj_b200_time_kernels(void* program, const void* const* inputs, void* const* outputs, void* stream,
                                int32_t iters, float* ms_per_kernel);

/* Synchronise the program's device and read its status words: code 0 = ok.
 * code/where receive the first failure recorded by a kernel (bounded wait
 * that ran out, or a checked-build bounds violation); the words are cleared. */
TJ_API int tj_b200_check_status(void* program, int32_t* code, int32_t* where);

/* Programmatic dependent launch between the program's kernels (enable != 0; the default unless
 * the environment sets TENSORJIT_B200_PDL=0): each kernel after the first may be scheduled while
 * the previous one finishes and waits (griddepcontrol.wait) before touching memory.  Saves launch
 * gaps in latency-bound programs; measured to cost clock under the power cap in programs of long
 * persistent GEMMs, so the Python front end enables it per program.  No counterpart in the
 * reference (its driver launches kernels in plain stream order, `cuda_driver.py:115-124`). */
TJ_API int tj_b200_set_pdl(void* program, int32_t enable);

TJ_API int tj_b200_program_info(void* program, tj_program_info* info);

TJ_API int tj_b200_destroy(void* program);

/* C[M,N] = A[M,K] * B[N,K]^T in f32 (row-major, contiguous, 16-byte aligned; K % 4 == 0),
 * computed as 3xTF32 on the tensor cores -- WITHOUT allocating any device memory.
 * No counterpart in the reference.  For callers that cannot call cudaMalloc: code inside a
 * host application that owns all device memory and hands out only input/output buffers,
 * and paths where an allocation could block or fail at the wrong moment.  Its workspace (the
 * TF32 hi/lo copies of A and B) is a static __device__ array of 4 x 2^21 floats (32 MiB,
 * held by every GPU that loads this library until exit): M*K and N*K must each be
 * <= 2097152, larger calls return TJ_ERR_INVALID.  All calls share that array, so calls
 * whose GPU work overlaps (different streams) race; serialise them.  The first call on a
 * device resolves the array's address (cudaGetSymbolAddress, that device current) and
 * should come before any stream capture.  `stream` is a cudaStream_t (NULL = legacy). */
TJ_API int tj_b200_linear_f32_noalloc(const float* A, const float* B, float* C, int32_t M, int32_t N, int32_t K,
                                      void* stream);

/* The failure record of tj_b200_linear_f32_noalloc on the current device.  Its GEMM's
 * waits are bounded: one that runs out makes the kernel give up and leave (code, site) in
 * status words that, like the scratch array, are static and shared by every call (each call
 * clears them when it starts).  This waits for `stream`, copies the words back, clears them
 * and returns TJ_OK with *code = 0 if the calls since the last read finished normally, else
 * TJ_ERR_DEVICE_STATUS with *code = 1 (wait timeout) and *where = the wait site.  Allocates
 * nothing.  No counterpart in the reference (its kernels have no bounded waits). */
TJ_API int tj_b200_linear_f32_noalloc_status(int32_t* code, int32_t* where, void* stream);

/* Peer memory between the processes of one node (one process per GPU), for row-sharded
 * programs whose output rows go straight into one rank's buffer over NVLink: the owner exports
 * the device allocation that holds `dptr`, every other rank opens it and passes the returned
 * address (plus its row offset) to tj_b200_run as an output pointer, so the program's last
 * kernel stores its rows into the owner's memory with no separate gather.
 * No counterpart in the reference (it runs on one device; its only output path is a copy,
 * `cuda_backend.py:535`).  A handle is the driver's 64-byte CUipcMemHandle; `offset` is
 * `dptr` minus the base of its allocation.  Allocations made through the virtual-memory API
 * (e.g. a caching allocator with expandable segments) cannot be exported: TJ_ERR_CUDA. */
typedef struct tj_ipc_handle {
  unsigned char bytes[64];
} tj_ipc_handle;

TJ_API int tj_b200_ipc_export(const void* dptr, int32_t device, tj_ipc_handle* handle, uint64_t* offset);

/* Map a handle exported by another process into this process on `device` (peer access is
 * enabled as needed); *dptr = mapped base + offset.  Release with tj_b200_ipc_close. */
TJ_API int tj_b200_ipc_open(const tj_ipc_handle* handle, uint64_t offset, int32_t device, void** dptr);

/* Unmap an address returned by tj_b200_ipc_open (same offset and device).  The caller must
 * have synchronised every stream that still writes through it. */
TJ_API int tj_b200_ipc_close(void* dptr, uint64_t offset, int32_t device);

/* Message of the last failure on this thread ("" if none). */
TJ_API const char* tj_b200_last_error(void);

TJ_API int tj_b200_abi_version(void);

/* 1 if libcuda can be loaded and reports at least one device, else 0. */
TJ_API int tj_b200_driver_available(void);

#ifdef __cplusplus
}
#endif

#endif /* TJ_B200_H */
