/*
 * A fake CUDA driver library for host-side failure injection (test fixture).
 *
 * libflight4s_b200.so opens it instead of libcuda.so.1 when
 * FLIGHT4S_CUDA_DRIVER names it.  It exports cuGetProcAddress_v2 and hands
 * out fakes for the driver entry points the library uses: contexts,
 * modules, functions, memory and streams are counters or malloc'd host
 * memory, kernel launches are recorded (function name, geometry, cluster
 * attribute, argument bytes) and never run.  Errors are injected by
 * environment:
 *   FAKE_CUDA_FAIL="cuLaunchKernelEx=719,cuMemAlloc=2"  entry point -> CUresult
 *   FAKE_CUDA_POP_MISMATCH=1   cuCtxPopCurrent reports a different context
 * Plays the role of the reference's RecordingBackend
 * (runtime/src/test/scala/flight4s/runtime/cuda/CudaResourcesSuite.scala)
 * one layer lower, under the native library.
 *
 * Build: gcc -O1 -fPIC -shared -I/usr/local/cuda/include fake_cuda.c -o libfakecuda.so
 */
#include <cuda.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------ injection */
static int injected(const char* fn) {
  const char* spec = getenv("FAKE_CUDA_FAIL");
  if (!spec) return 0;
  size_t len = strlen(fn);
  for (const char* p = spec; (p = strstr(p, fn)) != NULL; p += len) {
    if ((p == spec || p[-1] == ',') && p[len] == '=') return atoi(p + len + 1);
  }
  return 0;
}
#define INJECT(fn)                 \
  do {                             \
    int code_ = injected(#fn);     \
    if (code_) return (CUresult)code_; \
  } while (0)

/* ------------------------------------------------------------- recording */
typedef struct {
  char name[64];
  unsigned grid[3], block[3], smem;
  int cluster;
  unsigned cluster_dim[3];
  int nparams;
  unsigned char params[32][8];
  unsigned long long stream;
  int programmatic; /* CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION set */
} Launch;

static Launch last_launch;
static int launch_count;
#define HISTORY 64
static Launch history[HISTORY]; /* launch i (0-based since reset) at history[i % HISTORY] */

typedef struct {
  const char* name;
  int n;
  unsigned char sizes[16];
} Signature;

/* argument byte sizes of the kernels whose launches the tests inspect */
static const Signature signatures[] = {
    {"f4s_vector_add_f32", 4, {8, 8, 8, 4}},
    {"f4s_vector_add_bf16", 4, {8, 8, 8, 4}},
    {"f4s_vector_add_f16", 4, {8, 8, 8, 4}},
    {"f4s_vector_add_f64", 4, {8, 8, 8, 4}},
    {"f4s_vector_add_i32", 4, {8, 8, 8, 4}},
    {"f4s_reduce_sum_f32", 8, {8, 4, 4, 8, 8, 4, 4, 4}},
    {"f4s_reduce_sum_i32", 8, {8, 4, 4, 8, 8, 4, 4, 4}},
    {"f4s_reduce_argmax_f32", 8, {8, 4, 4, 8, 8, 4, 4, 4}},
    {"f4s_block_reduce_sum_f32", 5, {8, 4, 8, 8, 8}},
    {"f4s_block_sum_tiles_f32", 3, {8, 4, 8}},
    {"f4s_block_sum_upper_f32", 3, {8, 4, 8}},
    {"f4s_softmax_rows_bf16_v4", 4, {8, 8, 4, 4}},
    {"f4s_softmax_rows_bf16_any", 4, {8, 8, 4, 4}},
    {"f4s_rmsnorm_rows_bf16_tma", 6, {8, 8, 8, 4, 4, 4}},
    {"f4s_rmsnorm_rows_bf16_v8", 6, {8, 8, 8, 4, 4, 4}},
    {"f4s_rmsnorm_rows_bf16_any", 6, {8, 8, 8, 4, 4, 4}},
    {"f4s_fp8_quant_flat", 4, {8, 8, 8, 4}},
    {"f4s_fp8_quant_rows", 5, {8, 8, 8, 4, 4}},
    {"f4s_fp8_dequant_flat", 4, {8, 8, 8, 4}},
    {"f4s_convert_f32_f16_ru", 4, {8, 8, 4, 4}},
    {"f4s_convert_f32_bf16_rd", 4, {8, 8, 4, 4}},
    {"f4s_convert_f32_e4m3_sat", 4, {8, 8, 4, 4}},
    {"f4s_convert_f32_e5m2_nosat", 4, {8, 8, 4, 4}},
    {"f4s_convert_e5m2_f32", 4, {8, 8, 4, 4}},
    {"f4s_convert_copy_8", 4, {8, 8, 4, 4}},
    {"f4s_convert_copy_1", 4, {8, 8, 4, 4}},
    {"f4s_reduce_ordered_f32", 7, {8, 4, 4, 8, 8, 8, 4}},
    {"f4s_reduce_ordered_final", 5, {8, 4, 4, 8, 4}},
    {"write_values", 2, {8, 4}},
};

typedef struct {
  char name[64];
} FakeFunction;

/* exported for the tests */
int fake_launch_count(void) { return launch_count; }
const void* fake_last_launch(void) { return &last_launch; }
const void* fake_launch_at(int i) {
  return (i < 0 || i >= launch_count || i + HISTORY < launch_count) ? NULL : &history[i % HISTORY];
}
void fake_reset(void) {
  memset(&last_launch, 0, sizeof last_launch);
  launch_count = 0;
}

/* ---------------------------------------------------------------- state */
static int ctx_object, module_object, stream_object, event_object;
static CUcontext ctx_stack[64];
static int ctx_depth;
static CUdeviceptr next_address = 0x100000000ull;

/* ----------------------------------------------------------------- fakes */
static CUresult f_init(unsigned int flags) { (void)flags; INJECT(cuInit); return CUDA_SUCCESS; }

static const char* code_name(CUresult r) {
  switch ((int)r) {
    case 0: return "CUDA_SUCCESS";
    case 1: return "CUDA_ERROR_INVALID_VALUE";
    case 2: return "CUDA_ERROR_OUT_OF_MEMORY";
    case 201: return "CUDA_ERROR_INVALID_CONTEXT";
    case 218: return "CUDA_ERROR_INVALID_PTX";
    case 700: return "CUDA_ERROR_ILLEGAL_ADDRESS";
    case 719: return "CUDA_ERROR_LAUNCH_FAILED";
    default: return NULL;
  }
}
static CUresult f_err_name(CUresult e, const char** s) {
  *s = code_name(e);
  return *s ? CUDA_SUCCESS : CUDA_ERROR_INVALID_VALUE;
}
static CUresult f_err_string(CUresult e, const char** s) {
  *s = code_name(e) ? "fake driver error description" : NULL;
  return *s ? CUDA_SUCCESS : CUDA_ERROR_INVALID_VALUE;
}
static CUresult f_device_get(CUdevice* d, int ordinal) {
  INJECT(cuDeviceGet);
  if (ordinal != 0) return CUDA_ERROR_INVALID_DEVICE;
  *d = 0;
  return CUDA_SUCCESS;
}
static CUresult f_device_count(int* n) { *n = 1; return CUDA_SUCCESS; }
static CUresult f_device_attr(int* v, CUdevice_attribute a, CUdevice d) {
  (void)d;
  switch (a) {
    case CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MAJOR: *v = 10; break;
    case CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MINOR: *v = 0; break;
    case CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT: *v = 148; break;
    default: *v = 0;
  }
  return CUDA_SUCCESS;
}
static CUresult f_primary_retain(CUcontext* c, CUdevice d) {
  (void)d;
  INJECT(cuDevicePrimaryCtxRetain);
  *c = (CUcontext)&ctx_object;
  return CUDA_SUCCESS;
}
static CUresult f_primary_release(CUdevice d) { (void)d; return CUDA_SUCCESS; }
static CUresult f_push(CUcontext c) {
  INJECT(cuCtxPushCurrent);
  if (ctx_depth >= 64) return CUDA_ERROR_INVALID_VALUE;
  ctx_stack[ctx_depth++] = c;
  return CUDA_SUCCESS;
}
static CUresult f_pop(CUcontext* c) {
  if (ctx_depth == 0) return CUDA_ERROR_INVALID_CONTEXT;
  CUcontext top = ctx_stack[--ctx_depth];
  *c = getenv("FAKE_CUDA_POP_MISMATCH") ? (CUcontext)&module_object : top;
  return CUDA_SUCCESS;
}
static CUresult f_get_current(CUcontext* c) { *c = ctx_depth ? ctx_stack[ctx_depth - 1] : NULL; return CUDA_SUCCESS; }
static CUresult f_set_current(CUcontext c) {
  if (ctx_depth == 0) ctx_stack[ctx_depth++] = c; else ctx_stack[ctx_depth - 1] = c;
  return CUDA_SUCCESS;
}
static CUresult f_ctx_device(CUdevice* d) { *d = 0; return CUDA_SUCCESS; }
static CUresult f_ctx_id(CUcontext c, unsigned long long* id) { *id = (unsigned long long)(uintptr_t)c; return CUDA_SUCCESS; }
static CUresult f_stream_capturing(CUstream s, CUstreamCaptureStatus* st) { (void)s; *st = CU_STREAM_CAPTURE_STATUS_NONE; return CUDA_SUCCESS; }
static CUresult f_ctx_sync(void) { INJECT(cuCtxSynchronize); return CUDA_SUCCESS; }
static CUresult f_module_load(CUmodule* m, const void* image, unsigned n, CUjit_option* opts, void** vals) {
  (void)image;
  int code = injected("cuModuleLoadDataEx");
  if (code) {
    for (unsigned i = 0; i < n; ++i) {
      if (opts[i] == CU_JIT_ERROR_LOG_BUFFER) snprintf((char*)vals[i], 64, "fake error log");
    }
    return (CUresult)code;
  }
  *m = (CUmodule)&module_object;
  return CUDA_SUCCESS;
}
static CUresult f_module_unload(CUmodule m) { (void)m; return CUDA_SUCCESS; }
static CUresult f_get_function(CUfunction* f, CUmodule m, const char* name) {
  (void)m;
  INJECT(cuModuleGetFunction);
  FakeFunction* fn = (FakeFunction*)calloc(1, sizeof(FakeFunction));
  snprintf(fn->name, sizeof fn->name, "%s", name);
  *f = (CUfunction)fn;
  return CUDA_SUCCESS;
}
static unsigned int fake_global;
static CUresult f_get_global(CUdeviceptr* p, size_t* bytes, CUmodule m, const char* name) {
  (void)m; (void)name;
  *p = (CUdeviceptr)(uintptr_t)&fake_global;
  *bytes = sizeof fake_global;
  return CUDA_SUCCESS;
}
static CUresult f_func_attr(int* v, CUfunction_attribute a, CUfunction f) {
  (void)f;
  *v = (a == CU_FUNC_ATTRIBUTE_MAX_THREADS_PER_BLOCK) ? 1024 : (a == CU_FUNC_ATTRIBUTE_NUM_REGS ? 32 : 0);
  return CUDA_SUCCESS;
}
static CUresult f_func_set_attr(CUfunction f, CUfunction_attribute a, int v) { (void)f; (void)a; (void)v; return CUDA_SUCCESS; }
static CUresult f_occ_clusters(int* n, CUfunction f, const CUlaunchConfig* c) { (void)f; (void)c; *n = 37; return CUDA_SUCCESS; }
static CUresult f_occ_blocks(int* n, CUfunction f, int b, size_t s) { (void)f; (void)b; (void)s; *n = 4; return CUDA_SUCCESS; }
static CUresult f_stream_create(CUstream* s, unsigned flags) { (void)flags; *s = (CUstream)&stream_object; return CUDA_SUCCESS; }
static CUresult f_stream_destroy(CUstream s) { (void)s; return CUDA_SUCCESS; }
static CUresult f_stream_sync(CUstream s) { (void)s; INJECT(cuStreamSynchronize); return CUDA_SUCCESS; }
static CUresult f_stream_wait(CUstream s, CUevent e, unsigned f) { (void)s; (void)e; (void)f; return CUDA_SUCCESS; }
static CUresult f_event_create(CUevent* e, unsigned f) { (void)f; *e = (CUevent)&event_object; return CUDA_SUCCESS; }
static CUresult f_event_destroy(CUevent e) { (void)e; return CUDA_SUCCESS; }
static CUresult f_event_record(CUevent e, CUstream s) { (void)e; (void)s; return CUDA_SUCCESS; }
static CUresult f_event_query(CUevent e) { (void)e; return CUDA_ERROR_NOT_READY; }
static CUresult f_event_sync(CUevent e) { (void)e; return CUDA_SUCCESS; }
static CUresult f_event_elapsed(float* ms, CUevent a, CUevent b) { (void)a; (void)b; *ms = 1.5f; return CUDA_SUCCESS; }
static CUresult f_host_alloc(void** p, size_t n, unsigned f) {
  (void)f;
  INJECT(cuMemHostAlloc);
  *p = calloc(1, n ? n : 1);
  return *p ? CUDA_SUCCESS : CUDA_ERROR_OUT_OF_MEMORY;
}
static CUresult f_host_free(void* p) { free(p); return CUDA_SUCCESS; }
static CUresult f_alloc(CUdeviceptr* p, size_t n) {
  INJECT(cuMemAlloc);
  *p = next_address;
  next_address += (n + 511) / 512 * 512 + 512;
  return CUDA_SUCCESS;
}
static CUresult f_free(CUdeviceptr p) { (void)p; return CUDA_SUCCESS; }
static CUresult f_htod(CUdeviceptr d, const void* s, size_t n) { (void)d; (void)s; (void)n; INJECT(cuMemcpyHtoD); return CUDA_SUCCESS; }
static CUresult f_htod_async(CUdeviceptr d, const void* s, size_t n, CUstream st) { (void)d; (void)s; (void)n; (void)st; return CUDA_SUCCESS; }
static CUresult f_dtoh(void* d, CUdeviceptr s, size_t n) { (void)s; INJECT(cuMemcpyDtoH); memset(d, 0, n); return CUDA_SUCCESS; }
static CUresult f_dtoh_async(void* d, CUdeviceptr s, size_t n, CUstream st) { (void)s; (void)st; memset(d, 0, n); return CUDA_SUCCESS; }
static CUresult f_memset_async(CUdeviceptr d, unsigned char v, size_t n, CUstream s) { (void)d; (void)v; (void)n; (void)s; return CUDA_SUCCESS; }

static CUresult f_launch(const CUlaunchConfig* c, CUfunction f, void** params, void** extra) {
  (void)extra;
  INJECT(cuLaunchKernelEx);
  memset(&last_launch, 0, sizeof last_launch);
  const FakeFunction* fn = (const FakeFunction*)f;
  snprintf(last_launch.name, sizeof last_launch.name, "%s", fn->name);
  last_launch.grid[0] = c->gridDimX; last_launch.grid[1] = c->gridDimY; last_launch.grid[2] = c->gridDimZ;
  last_launch.block[0] = c->blockDimX; last_launch.block[1] = c->blockDimY; last_launch.block[2] = c->blockDimZ;
  last_launch.smem = c->sharedMemBytes;
  last_launch.stream = (unsigned long long)(uintptr_t)c->hStream;
  for (unsigned i = 0; i < c->numAttrs; ++i) {
    if (c->attrs[i].id == CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION)
      last_launch.programmatic = c->attrs[i].value.programmaticStreamSerializationAllowed != 0;
    if (c->attrs[i].id == CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION) {
      last_launch.cluster = 1;
      last_launch.cluster_dim[0] = c->attrs[i].value.clusterDim.x;
      last_launch.cluster_dim[1] = c->attrs[i].value.clusterDim.y;
      last_launch.cluster_dim[2] = c->attrs[i].value.clusterDim.z;
    }
  }
  for (size_t s = 0; s < sizeof signatures / sizeof signatures[0]; ++s) {
    if (strcmp(signatures[s].name, fn->name) == 0 && params != NULL) {
      last_launch.nparams = signatures[s].n;
      for (int i = 0; i < signatures[s].n; ++i) memcpy(last_launch.params[i], params[i], signatures[s].sizes[i]);
    }
  }
  history[launch_count % HISTORY] = last_launch;
  ++launch_count;
  return CUDA_SUCCESS;
}

/* -------------------------------------------------------- proc addresses */
typedef struct {
  const char* name;
  void* fn;
} Entry;

static const Entry entries[] = {
    {"cuInit", (void*)f_init},
    {"cuGetErrorName", (void*)f_err_name},
    {"cuGetErrorString", (void*)f_err_string},
    {"cuDeviceGet", (void*)f_device_get},
    {"cuDeviceGetCount", (void*)f_device_count},
    {"cuDeviceGetAttribute", (void*)f_device_attr},
    {"cuDevicePrimaryCtxRetain", (void*)f_primary_retain},
    {"cuDevicePrimaryCtxRelease", (void*)f_primary_release},
    {"cuCtxPushCurrent", (void*)f_push},
    {"cuCtxPopCurrent", (void*)f_pop},
    {"cuCtxGetCurrent", (void*)f_get_current},
    {"cuCtxSetCurrent", (void*)f_set_current},
    {"cuCtxGetDevice", (void*)f_ctx_device},
    {"cuCtxGetId", (void*)f_ctx_id},
    {"cuCtxSynchronize", (void*)f_ctx_sync},
    {"cuModuleLoadDataEx", (void*)f_module_load},
    {"cuModuleUnload", (void*)f_module_unload},
    {"cuModuleGetFunction", (void*)f_get_function},
    {"cuModuleGetGlobal", (void*)f_get_global},
    {"cuFuncGetAttribute", (void*)f_func_attr},
    {"cuFuncSetAttribute", (void*)f_func_set_attr},
    {"cuOccupancyMaxActiveClusters", (void*)f_occ_clusters},
    {"cuOccupancyMaxActiveBlocksPerMultiprocessor", (void*)f_occ_blocks},
    {"cuStreamCreate", (void*)f_stream_create},
    {"cuStreamDestroy", (void*)f_stream_destroy},
    {"cuStreamSynchronize", (void*)f_stream_sync},
    {"cuStreamWaitEvent", (void*)f_stream_wait},
    {"cuStreamIsCapturing", (void*)f_stream_capturing},
    {"cuEventCreate", (void*)f_event_create},
    {"cuEventDestroy", (void*)f_event_destroy},
    {"cuEventRecord", (void*)f_event_record},
    {"cuEventQuery", (void*)f_event_query},
    {"cuEventSynchronize", (void*)f_event_sync},
    {"cuEventElapsedTime", (void*)f_event_elapsed},
    {"cuMemHostAlloc", (void*)f_host_alloc},
    {"cuMemFreeHost", (void*)f_host_free},
    {"cuMemAlloc", (void*)f_alloc},
    {"cuMemFree", (void*)f_free},
    {"cuMemcpyHtoD", (void*)f_htod},
    {"cuMemcpyHtoDAsync", (void*)f_htod_async},
    {"cuMemcpyDtoH", (void*)f_dtoh},
    {"cuMemcpyDtoHAsync", (void*)f_dtoh_async},
    {"cuMemsetD8Async", (void*)f_memset_async},
    {"cuLaunchKernelEx", (void*)f_launch},
};

__attribute__((visibility("default"))) CUresult cuGetProcAddress_v2(const char* symbol, void** pfn, int version,
                                                                  cuuint64_t flags,
                                                                  CUdriverProcAddressQueryResult* status) {
  (void)version; (void)flags;
  for (size_t i = 0; i < sizeof entries / sizeof entries[0]; ++i) {
    if (strcmp(entries[i].name, symbol) == 0) {
      *pfn = entries[i].fn;
      if (status) *status = CU_GET_PROC_ADDRESS_SUCCESS;
      return CUDA_SUCCESS;
    }
  }
  *pfn = NULL;
  if (status) *status = CU_GET_PROC_ADDRESS_SYMBOL_NOT_FOUND;
  return CUDA_ERROR_NOT_FOUND;
}
