/*
 * drift_runtime.h -- the runtime half of libdrift_cuda's C ABI.
 *
 * The drift runner's host reaches its GPU through hand-written FFM bindings to
 * a few dozen libamdhip64 functions (runner/src/drift/runner/native/
 * HipRuntime.scala:73-120) and launches kernels by name out of loaded code
 * objects (native/KernelModule.scala:8-33, HipRuntime.scala:310-363). These
 * entry points are their CUDA-side replacements, one for one, with the same
 * argument meanings: every function returns an int status (0 = success, a
 * cudaError_t value for a CUDA failure, or DRIFT_ERROR_INVALID_ARGUMENT for an
 * argument the library refuses), out-parameters are pointer slots, device
 * pointers are plain addresses the host never dereferences.
 *
 * Only plain C types appear here: the header is what a JDK FFM (Panama)
 * binding, a ctypes stub or C code includes.
 */
#ifndef DRIFT_RUNTIME_H
#define DRIFT_RUNTIME_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* An argument the library refuses (a failed `require` in the reference:
 * runner/src/drift/runner/ops/Ops.scala:36-93); the message says which. */
#define DRIFT_ERROR_INVALID_ARGUMENT 1001
/* A bounded device-side wait gave up (no reference counterpart: the
 * reference's spin waits never time out, kernels/matvec.hip:1785-1787). */
#define DRIFT_ERROR_TIMEOUT 1002

typedef void* drift_stream_t;   /* a cudaStream_t; NULL is the legacy default stream */
typedef void* drift_event_t;    /* a cudaEvent_t */
typedef void* drift_module_t;   /* a loaded kernel image; NULL names this library's own kernels */
typedef void* drift_function_t; /* a kernel in a module */

/* hipInit (HipRuntime.scala:73): initialises the runtime; flags must be 0. */
int drift_init(int flags);
/* hipSetDevice (HipRuntime.scala:74): this thread's device. */
int drift_set_device(int device);
/* hipGetDevice: this thread's device (new: one process or thread per GPU). */
int drift_get_device(int* device);
/* hipGetDeviceCount (new: the reference pins device 0, HipRuntime.scala:149-150). */
int drift_get_device_count(int* count);
/* hipSetDeviceFlags (HipRuntime.scala:75, 152-165): 1 spin, 2 yield, 4 blocking sync. */
int drift_set_device_flags(int flags);
/* hipDeviceGetName (HipRuntime.scala:76-77). */
int drift_device_get_name(char* name, int length, int device);
/* hipDeviceSynchronize (HipRuntime.scala:78). */
int drift_device_synchronize(void);
/* hipMemGetInfo (HipRuntime.scala:79). */
int drift_mem_get_info(size_t* free_bytes, size_t* total_bytes);
/* hipGetErrorString (HipRuntime.scala:80-81): the text of a status this
 * library returned; for DRIFT_ERROR_* codes, the calling thread's last message. */
const char* drift_get_error_string(int status);
/* The calling thread's last error message, or "" (new). */
const char* drift_last_error_message(void);

/* hipMalloc / hipFree / hipMemset (HipRuntime.scala:82-84). */
int drift_malloc(void** pointer, size_t bytes);
int drift_free(void* pointer);
int drift_memset(void* pointer, int value, size_t bytes);
/* hipMemcpy / hipMemcpyAsync (HipRuntime.scala:85-88); kind 4 = default
 * (the direction follows from the addresses), as MemcpyDefault (L372-373). */
int drift_memcpy(void* target, const void* source, size_t bytes, int kind);
int drift_memcpy_async(void* target, const void* source, size_t bytes, int kind,
                       drift_stream_t stream);
/* hipHostRegister / hipHostUnregister / hipHostGetDevicePointer
 * (HipRuntime.scala:89-93); flags as hipHostRegisterMapped (2) / ReadOnly (8). */
int drift_host_register(void* host, size_t bytes, int flags);
int drift_host_unregister(void* host);
int drift_host_get_device_pointer(void** device, void* host, int flags);

/* hipStreamCreate / Destroy / Synchronize (HipRuntime.scala:94-96). */
int drift_stream_create(drift_stream_t* stream);
int drift_stream_destroy(drift_stream_t stream);
int drift_stream_synchronize(drift_stream_t stream);

/* hipEventCreate / Destroy / Record / Synchronize / ElapsedTime
 * (HipRuntime.scala:97-102). */
int drift_event_create(drift_event_t* event);
int drift_event_destroy(drift_event_t event);
int drift_event_record(drift_event_t event, drift_stream_t stream);
int drift_event_synchronize(drift_event_t event);
int drift_event_elapsed_time(float* milliseconds, drift_event_t start, drift_event_t end);
/* New (the reference's binding has no counterpart; hipStreamWaitEvent is the
 * HIP call): work queued on `stream` after this waits for the event's last
 * record -- how a host overlaps copies on one stream with products on
 * another. */
int drift_stream_wait_event(drift_stream_t stream, drift_event_t event);

/* hipModuleLoadData / Unload / GetFunction (HipRuntime.scala:103-106): a cubin
 * or fatbin image built for sm_100a. drift_module_get_function with module NULL
 * finds a kernel of this library by its extern "C" name (drift_kernels.h). */
int drift_module_load_data(drift_module_t* module, const void* image);
int drift_module_unload(drift_module_t module);
int drift_module_get_function(drift_function_t* function, drift_module_t module,
                              const char* name);

/* hipModuleLaunchKernel (HipRuntime.scala:107-119, 310-363): kernel_params is
 * an array of pointers to the argument values, as the reference packs them;
 * extra must be NULL. */
int drift_module_launch_kernel(drift_function_t function, unsigned grid_x, unsigned grid_y,
                               unsigned grid_z, unsigned block_x, unsigned block_y,
                               unsigned block_z, unsigned shared_bytes, drift_stream_t stream,
                               void** kernel_params, void** extra);

/* The number of kernels this library holds, and the name of kernel i: what a
 * host lists to check its by-name table (new). */
int drift_kernel_count(void);
const char* drift_kernel_name(int index);

#ifdef __cplusplus
}
#endif

#endif /* DRIFT_RUNTIME_H */
