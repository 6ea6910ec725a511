/*
 * flight4s_b200 — C ABI of the B200 (sm_100a) hot path.
 *
 * Two groups of entry points:
 *
 *  1. The runtime boundary.  One plain-C function per native method the
 *     reference's JVM runtime binds (runtime/src/main/java/flight4s/runtime/
 *     cuda/internal/CudaNativeBindings.java:21-151, implemented in
 *     native/src/jni_cuda_launcher.cpp and native/src/jni_cuda_driver.cpp).
 *     Handles travel as uint64_t exactly as the JNI layer passes them as
 *     `long`; byte arrays and direct buffers become pointer + size.
 *
 *  2. The hot-path operators: the sm_100a kernels that replace the
 *     reference's serial `ReduceSum` lowering
 *     (core/src/main/scala/flight4s/core/codegen/CudaCodegen.scala:383-403),
 *     its `vectorAdd` / `blockReduceSum` test kernels
 *     (runtime/src/test/scala/flight4s/runtime/cuda/CudaResourcesJniSuite.scala:108-312)
 *     and the row-wise / FP8 ops.  They run on an `f4s_hotpath`, which holds
 *     the embedded sm_100a module loaded into one context.  The kernels are
 *     also ordinary module functions: f4s_hotpath_module() + f4s_resolve_function()
 *     + f4s_launch_kernel() launch them through the same descriptor-coded
 *     path as any user kernel.
 *
 * Status convention (every function returning int):
 *     0                           success
 *     > 0                         a CUresult from the CUDA driver
 *     F4S_STATUS_INVALID_ARGUMENT the request was rejected before reaching
 *                                 the driver (the reference throws
 *                                 std::invalid_argument -> IllegalArgumentException)
 *     F4S_STATUS_OVERFLOW         a size or offset overflowed (std::overflow_error)
 *     F4S_STATUS_DRIVER_UNAVAILABLE libcuda.so.1 could not be loaded
 *     F4S_STATUS_INTERNAL         any other native failure
 * The calling thread's last status (name, description, and the module-load
 * JIT logs the reference returns in NativeCudaDriverResult) is available
 * from f4s_last_status_*() until the thread's next call.
 *
 * Nothing here synchronizes unless its comment says so.
 */
#ifndef FLIGHT4S_B200_H_
#define FLIGHT4S_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define F4S_STATUS_SUCCESS 0
#define F4S_STATUS_INVALID_ARGUMENT (-1)
#define F4S_STATUS_OVERFLOW (-2)
#define F4S_STATUS_DRIVER_UNAVAILABLE (-3)
#define F4S_STATUS_INTERNAL (-4)

/* ------------------------------------------------------------- diagnostics */

/* ABI version of this header (major * 1000 + minor). */
int f4s_abi_version(void);

/* Last status of the calling thread: code, CUDA name (e.g. "CUDA_SUCCESS",
 * "CUDA_ERROR_INVALID_VALUE") or exception text, description, JIT logs.
 * Fields of NativeCudaDriverResult (NativeCudaDriverResult.java). */
int f4s_last_status_code(void);
const char* f4s_last_status_name(void);
const char* f4s_last_status_description(void);
const char* f4s_last_info_log(void);
const char* f4s_last_error_log(void);

/* 1 when libcuda.so.1 loads on this host, else 0 (and the reason in
 * f4s_last_status_description()).  Never touches a device. */
int f4s_driver_available(void);

/* ------------------------------------------------------- launch contract */

/* Launch geometry and argument layout checks of the reference's contract
 * (native/include/flight4s/cuda/launch_contract.hpp:35-42,
 * native/src/launch_contract.cpp:49-199).  Return 0 when valid, else
 * F4S_STATUS_INVALID_ARGUMENT with the reference's message in
 * f4s_last_status_description().  Pure host code: no driver needed.
 * Descriptor codes are the reference's 1..10 (1 bool, 2 i32, 3 u32, 4 f16,
 * 5 bf16, 6 f32, 7 f64, 8 e4m3, 9 e5m2, 10 device pointer;
 * core/src/main/scala/flight4s/core/abi/CudaAbi.scala:11-20) plus one
 * addition, 11 = signed 64-bit integer (8 bytes, 8-aligned), for element
 * counts and offsets above 2^31 - 1; every other code is rejected with the
 * reference's message. */
int f4s_validate_launch_geometry(int32_t grid_x, int32_t grid_y, int32_t grid_z, int32_t block_x,
                                 int32_t block_y, int32_t block_z, int32_t dynamic_shared_memory_bytes,
                                 int32_t uses_cluster, int32_t cluster_x, int32_t cluster_y,
                                 int32_t cluster_z);
int f4s_validate_argument_layout(const void* storage, int64_t storage_size_bytes, const int32_t* offsets,
                                 size_t offset_count, const int8_t* descriptor_codes,
                                 size_t descriptor_count);

/* Replaces CudaNativeBindings.launchKernel (CudaNativeBindings.java:21-38;
 * native/src/jni_cuda_launcher.cpp:155-203 -> CudaLauncher::launch,
 * native/src/cuda_launcher.cpp:8-62).  `argument_storage` holds the packed
 * arguments at `argument_offsets` with `argument_descriptor_codes`
 * (bool 1, i32 2, u32 3, f16 4, bf16 5, f32 6, f64 7, e4m3 8, e5m2 9,
 * device pointer 10).  Pushes `context`, calls cuLaunchKernelEx (with the
 * cluster attribute when uses_cluster != 0), restores the caller's context. */
int f4s_launch_kernel(uint64_t context, uint64_t function, uint64_t stream, int32_t grid_x,
                      int32_t grid_y, int32_t grid_z, int32_t block_x, int32_t block_y, int32_t block_z,
                      int32_t dynamic_shared_memory_bytes, int32_t uses_cluster, int32_t cluster_x,
                      int32_t cluster_y, int32_t cluster_z, void* argument_storage,
                      int64_t argument_storage_size_bytes, const int32_t* argument_offsets,
                      const int8_t* argument_descriptor_codes, size_t argument_count);

/* ------------------------------------------------------------- contexts */

/* Replaces retainPrimaryContext (CudaNativeBindings.java:47-48;
 * native/src/jni_cuda_driver.cpp:427; native/src/cuda_driver.cpp:137-182). */
int f4s_retain_primary_context(int32_t device_ordinal, uint64_t* context, int32_t* compute_capability_major,
                               int32_t* compute_capability_minor);
/* Replaces releasePrimaryContext (CudaNativeBindings.java:50-51; native/src/jni_cuda_driver.cpp:446). */
int f4s_release_primary_context(int32_t device_ordinal);
/* Replaces synchronizeContext (CudaNativeBindings.java:53-54; native/src/jni_cuda_driver.cpp:465).  Synchronizes. */
int f4s_synchronize_context(uint64_t context);
/* Addition: cuDeviceGetAttribute for the context's device. */
int f4s_device_attribute(uint64_t context, int32_t attribute, int32_t* value);

/* -------------------------------------------------------------- modules */

/* Replaces loadPtx (CudaNativeBindings.java:56-58; native/src/jni_cuda_driver.cpp:484;
 * native/src/cuda_driver.cpp:209-261):
 * NUL-free PTX text, JIT logs in f4s_last_info_log()/f4s_last_error_log(). */
int f4s_load_ptx(uint64_t context, const uint8_t* ptx, size_t ptx_size, uint64_t* module);
/* Addition: load a cubin or fatbin image (the PTX path rejects NUL bytes,
 * native/src/cuda_driver.cpp:214-216, so it cannot carry sm_100a binaries). */
int f4s_load_module_image(uint64_t context, const void* image, size_t image_size, uint64_t* module);
/* Replaces unloadModule (CudaNativeBindings.java:60-62; native/src/jni_cuda_driver.cpp:504). */
int f4s_unload_module(uint64_t context, uint64_t module);
/* Replaces resolveFunction (CudaNativeBindings.java:64-67; native/src/jni_cuda_driver.cpp:524). */
int f4s_resolve_function(uint64_t context, uint64_t module, const char* name, uint64_t* function);
/* Replaces queryFunctionAttributes (CudaNativeBindings.java:69-71; native/src/jni_cuda_driver.cpp:548);
 * attributes = {max threads per block, static smem, const bytes, local
 * bytes, registers per thread}. */
int f4s_query_function_attributes(uint64_t context, uint64_t function, int32_t attributes[5]);

/* ------------------------------------------------------ streams, events */

/* Replace createStream / destroyStream / synchronizeStream
 * (CudaNativeBindings.java:73-83; native/src/jni_cuda_driver.cpp:568-627); flags 0
 * (default) or 1 (non-blocking). */
int f4s_create_stream(uint64_t context, int32_t flags, uint64_t* stream);
int f4s_destroy_stream(uint64_t context, uint64_t stream);
int f4s_synchronize_stream(uint64_t context, uint64_t stream);

/* Replace createEvent / destroyEvent / recordEvent / queryEvent /
 * synchronizeEvent / waitForEvent (CudaNativeBindings.java:85-109;
 * native/src/jni_cuda_driver.cpp:628-749); flags
 * may combine 1 (blocking sync) and 2 (disable timing). */
int f4s_create_event(uint64_t context, int32_t flags, uint64_t* event);
int f4s_destroy_event(uint64_t context, uint64_t event);
int f4s_record_event(uint64_t context, uint64_t event, uint64_t stream);
int f4s_query_event(uint64_t context, uint64_t event, int32_t* complete);
int f4s_synchronize_event(uint64_t context, uint64_t event);
int f4s_wait_for_event(uint64_t context, uint64_t stream, uint64_t event);
/* Addition: elapsed milliseconds between two recorded timing events (the
 * reference's event modes all disable timing, CudaResources.scala:104-106). */
int f4s_event_elapsed_ms(uint64_t context, uint64_t start_event, uint64_t end_event, float* milliseconds);

/* --------------------------------------------------------------- memory */

/* Replace allocatePinnedMemory / freePinnedMemory / allocateDeviceMemory /
 * freeDeviceMemory (CudaNativeBindings.java:111-125; native/src/jni_cuda_driver.cpp:750-829). */
int f4s_allocate_pinned_memory(uint64_t context, uint64_t size_bytes, void** host_address);
int f4s_free_pinned_memory(uint64_t context, void* host_address);
int f4s_allocate_device_memory(uint64_t context, uint64_t size_bytes, uint64_t* device_address);
int f4s_free_device_memory(uint64_t context, uint64_t device_address);

/* Replace copyHostToDevice(/Async) and copyDeviceToHost(/Async)
 * (CudaNativeBindings.java:127-151; native/src/jni_cuda_driver.cpp:830-935); the JNI direct buffer becomes
 * (host pointer, size_bytes).  The synchronous forms block. */
int f4s_copy_host_to_device(uint64_t context, uint64_t device_address, uint64_t device_offset_bytes,
                            const void* source, uint64_t size_bytes);
int f4s_copy_host_to_device_async(uint64_t context, uint64_t device_address, uint64_t device_offset_bytes,
                                  const void* source, uint64_t size_bytes, uint64_t stream);
int f4s_copy_device_to_host(uint64_t context, uint64_t device_address, uint64_t device_offset_bytes,
                            void* destination, uint64_t size_bytes);
int f4s_copy_device_to_host_async(uint64_t context, uint64_t device_address, uint64_t device_offset_bytes,
                                  void* destination, uint64_t size_bytes, uint64_t stream);

/* ------------------------------------------------------ hot-path module */

typedef struct f4s_hotpath f4s_hotpath;

/* Loads the embedded sm_100a module into `context` and sizes launch shapes
 * for its device.  The module is what `CudaContext.load` would return for
 * these kernels (runtime/src/main/scala/flight4s/runtime/cuda/CudaResources.scala:137-167). */
int f4s_hotpath_open(uint64_t context, f4s_hotpath** hotpath);
int f4s_hotpath_close(f4s_hotpath* hotpath);
/* Module handle, for f4s_resolve_function / f4s_launch_kernel. */
uint64_t f4s_hotpath_module(const f4s_hotpath* hotpath);
int f4s_hotpath_sm_count(const f4s_hotpath* hotpath);
/* CTAs per cluster of the full-array reductions (1..8, default 4). */
int f4s_hotpath_set_reduce_cluster(f4s_hotpath* hotpath, int32_t cluster);
/* Launch overlap of the device-resident full-array reductions
 * (f4s_reduce_sum_f32 / _i32 / _argmax_f32, f4s_reduce_sum, f4s_reduce_argmax,
 * f4s_reduce_sum_policy under Fast):
 * when enabled, each is launched as a programmatic dependent of the kernel
 * before it on the stream, so it starts reading its input while that kernel
 * finishes and waits for it only before writing its workspace and output.
 * Enable only when no kernel that writes a reduction's input is launched
 * immediately before that reduction on the same stream.  Off by default.
 * No counterpart in the reference (its launches are fully serialized). */
int f4s_hotpath_set_launch_overlap(f4s_hotpath* hotpath, int32_t enable);

/* Device-side waits never spin forever: a kernel that waits on a barrier
 * (the TMA-staged RMSNorm) gives up after a bounded number of polls,
 * leaves its remaining rows unwritten and counts the event.  This reads the
 * count (after synchronizing the context) and optionally clears it. */
int f4s_hotpath_wait_timeouts(f4s_hotpath* hotpath, uint32_t* count, int32_t reset);
/* Diagnostic: launches one thread that waits, bounded to `polls` polls, on
 * a barrier nothing will complete, so the give-up path runs on the device
 * and raises the count above.  Asynchronous on the legacy default stream. */
int f4s_hotpath_check_bounded_wait(f4s_hotpath* hotpath, uint32_t polls);

/* ---------------------------------------------- full-array reductions */

/* Workspace (device bytes) every reduction on this hotpath needs: a ticket
 * counter plus one 16-byte partial per cluster.  Allocate it once, zeroed;
 * each launch leaves it zeroed again.  Launches sharing one workspace must
 * be ordered (same stream or events). */
uint64_t f4s_reduce_workspace_bytes(const f4s_hotpath* hotpath);

/* Parallel lowering of the reference's `ReduceSum`
 * (core/src/main/scala/flight4s/core/ir/IR.scala:96-107) over in[0, n):
 *   sum_f32:    *out (f64) = sum in[i], f32 values accumulated in f64;
 *   sum_i32:    *out (i32) = sum in[i], two's-complement wrap (bit-exact);
 *   argmax_f32: out[0] (i64) = (signed totalOrder key of the max << 32) | (0xFFFFFFFF - index),
 *               so the int64 max of packed keys from several devices is again
 *               (max value, lowest index); INT64_MIN if n == 0;
 *               out[1] (i64) = index of the first maximum (+ index_base), -1 if n == 0.
 *               The totalOrder key is bits ^ ((bits >> 31) & 0x7FFFFFFF) read as i32.
 * With accumulate != 0 the result is combined with the value already in
 * `out` (chunked or sharded inputs).  One launch; asynchronous on `stream`. */
int f4s_reduce_sum_f32(f4s_hotpath* hotpath, uint64_t stream, uint64_t in, uint64_t n, uint64_t out,
                       uint64_t workspace, uint64_t workspace_bytes, int32_t accumulate);
int f4s_reduce_sum_i32(f4s_hotpath* hotpath, uint64_t stream, uint64_t in, uint64_t n, uint64_t out,
                       uint64_t workspace, uint64_t workspace_bytes, int32_t accumulate);
int f4s_reduce_argmax_f32(f4s_hotpath* hotpath, uint64_t stream, uint64_t in, uint64_t n, uint64_t out,
                          uint64_t workspace, uint64_t workspace_bytes, uint64_t index_base,
                          int32_t accumulate);

/* max / argmax over every OrderedType of the reference
 * (core/src/main/scala/flight4s/core/types/CudaType.scala:182-188) by
 * launch-ABI code: 2 i32, 3 u32, 4 f16, 5 bf16, 6 f32, 7 f64.  Order: the
 * integers' own; IEEE totalOrder for the floats (-NaN < -inf < ... < -0 <
 * +0 < ... < +inf < +NaN); ties to the lowest index.  The 16-byte record
 * is f4s_reduce_argmax_f32's, with the type's order key (i32: the value;
 * u32: bits ^ 0x80000000; f16 / bf16: bits ^ ((bits >> 15 & 1) * 0x7FFF),
 * sign-extended; f32: as above) packed in out[0] -- except f64, whose
 * 64-bit key (bits ^ ((bits >> 63 & 1) * 0x7FFF...F)) fills out[0] alone.
 * index_base / accumulate as f4s_reduce_argmax_f32. */
int f4s_reduce_argmax(f4s_hotpath* hotpath, uint64_t stream, int32_t input_type, uint64_t in, uint64_t n,
                      uint64_t out, uint64_t workspace, uint64_t workspace_bytes, uint64_t index_base,
                      int32_t accumulate);

/* ReduceSum over every input type the reference accumulates
 * (AccumulatorType, core/src/main/scala/flight4s/core/types/CudaType.scala:199-230),
 * selected by its launch-ABI type code
 * (core/src/main/scala/flight4s/core/abi/CudaAbi.scala:11-20):
 *   2 i32, 3 u32:  *out (4 bytes) = 32-bit two's-complement wrapping sum
 *                  (bit-exact; the reference accumulates I32 in I32, U32 in U32);
 *   4 f16, 5 bf16, 6 f32, 8 fp8 e4m3, 9 fp8 e5m2, 7 f64:
 *                  *out (f64) = sum of the exactly widened inputs, partial
 *                  sums of each 16-byte vector in f32 (f64 for f64 input),
 *                  everything above in f64 -- a wider accumulator than the
 *                  reference's F32 for the 16-bit and 8-bit inputs.
 * Other codes (1 bool, 10 pointer) return F4S_STATUS_INVALID_ARGUMENT.  `in`
 * is aligned to its element size.  Code 6 is f4s_reduce_sum_f32 and code 2
 * f4s_reduce_sum_i32.  One launch; asynchronous on `stream`. */
int f4s_reduce_sum(f4s_hotpath* hotpath, uint64_t stream, int32_t input_type, uint64_t in, uint64_t n,
                   uint64_t out, uint64_t workspace, uint64_t workspace_bytes, int32_t accumulate);

/* ReduceSum under the reference's ReductionPolicy
 * (core/src/main/scala/flight4s/core/ir/IR.scala:79-82): 0 Strict,
 * 1 Deterministic, 2 Fast.
 *   Fast: f4s_reduce_sum (partial sums associated by launch geometry:
 *         reproducible for one device and launch shape).
 *   Strict, Deterministic, floating-point inputs (f16 bf16 f32 f64 e4m3
 *         e5m2): order-fixed kernels.  The body (from the first 16-byte
 *         boundary) is cut into 256 KiB groups; every group's f64 partial is
 *         a fixed tree over its elements, the total is a fixed tree over the
 *         group partials plus the unaligned head elements in order.  The
 *         result depends on the elements and the 16-byte phase of `in`
 *         only: the same bits on any grid, cluster size, B200 or number of
 *         GPUs holding whole groups (f4s_reduce_ordered_final).  The
 *         reference's Strict names its serial loop's order, which no parallel
 *         sum keeps; Strict gets the same fixed order as Deterministic.
 *   Integer inputs are exact under every policy (Fast kernel).
 * The workspace needed depends on the policy and n:
 * f4s_reduce_policy_workspace_bytes.  Group partials (f64) stay readable in
 * the workspace from byte 256 after an order-fixed launch. */
int f4s_reduce_sum_policy(f4s_hotpath* hotpath, uint64_t stream, int32_t input_type, int32_t policy, uint64_t in,
                          uint64_t n, uint64_t out, uint64_t workspace, uint64_t workspace_bytes,
                          int32_t accumulate);
int f4s_reduce_policy_workspace_bytes(const f4s_hotpath* hotpath, int32_t input_type, int32_t policy, uint64_t n,
                                      uint64_t* bytes);
/* Number of 256 KiB group partials an order-fixed sum of in[0, n) writes. */
int f4s_reduce_ordered_groups(int32_t input_type, uint64_t in, uint64_t n, uint64_t* groups);
/* *out (f64) = the order-fixed total of `count` group partials (f64, device
 * memory), e.g. the partials of several GPUs' shards concatenated in array
 * order.  One launch; asynchronous on `stream`. */
int f4s_reduce_ordered_final(f4s_hotpath* hotpath, uint64_t stream, uint64_t groups, uint64_t count, uint64_t out,
                             int32_t accumulate);

/* End-to-end form over a HOST buffer (pinned for overlap): chunked
 * host->device copies on `copy_stream` overlapped with the reduction on
 * `compute_stream` through `staging` (device, >= 768 bytes, 256-aligned),
 * result written to `host_out` (8 / 4 / 16 bytes as above; argmax indices
 * start at `index_base`).  op: 0 sum_f32, 1 sum_i32, 2 argmax_f32,
 * 3 sum_u32, 4 sum_f16, 5 sum_bf16, 6 sum_f64, 7 sum_e4m3, 8 sum_e5m2
 * (results as f4s_reduce_sum), 9 argmax_i32, 10 argmax_u32, 11 argmax_f16,
 * 12 argmax_bf16, 13 argmax_f64 (records as f4s_reduce_argmax).
 * Synchronizes both streams before returning. */
int f4s_reduce_host(f4s_hotpath* hotpath, int32_t op, const void* host_in, uint64_t n, uint64_t index_base,
                    void* host_out, uint64_t staging, uint64_t staging_bytes, uint64_t workspace,
                    uint64_t workspace_bytes, uint64_t copy_stream, uint64_t compute_stream);

/* The sum of a HOST buffer of any AdditiveType (input_type as
 * f4s_reduce_sum) under a ReductionPolicy (as f4s_reduce_sum_policy):
 * policy 2 Fast (and every integer sum) runs f4s_reduce_host's pipeline;
 * 0 Strict / 1 Deterministic floating-point sums stage chunks of whole
 * 256 KiB groups (staging >= 256 + 2 * 262144 bytes) and write each
 * group's partial to its place in `workspace`
 * (f4s_reduce_policy_workspace_bytes(n) bytes, ticket zeroed once), then
 * run F over all of them: the f64 result is bit-identical to
 * f4s_reduce_sum_policy over the same array at a 16-byte-aligned device
 * address, whatever the staging size.  Synchronizes both streams before
 * returning. */
int f4s_reduce_host_sum_policy(f4s_hotpath* hotpath, int32_t input_type, int32_t policy, const void* host_in,
                               uint64_t n, void* host_out, uint64_t staging, uint64_t staging_bytes,
                               uint64_t workspace, uint64_t workspace_bytes, uint64_t copy_stream,
                               uint64_t compute_stream);

/* The same pipeline computing the f32 sum and the argmax of one host array
 * from a single host->device transfer of each chunk (the two reductions
 * share every staged chunk): host_sum_out receives 8 bytes, host_argmax_out
 * 16 bytes, as above.  Synchronizes both streams before returning. */
int f4s_reduce_host_sum_argmax_f32(f4s_hotpath* hotpath, const void* host_in, uint64_t n, uint64_t index_base,
                                   void* host_sum_out, void* host_argmax_out, uint64_t staging,
                                   uint64_t staging_bytes, uint64_t workspace, uint64_t workspace_bytes,
                                   uint64_t copy_stream, uint64_t compute_stream);

/* -------------------------------------------------------------- Convert */

/* The reference's Convert node (core/src/main/scala/flight4s/core/ir/IR.scala:54-70)
 * over n elements, out[i] = convert(in[i]), types by launch-ABI code:
 *   6 f32 -> 4 f16 / 5 bf16: rounding 0 NearestEven, 1 TowardZero,
 *        2 TowardPositive, 3 TowardNegative (__float2half_{rn,rz,ru,rd},
 *        __float2bfloat16_{rn,rz,ru,rd});
 *   6 f32 -> 8 e4m3 / 9 e5m2: saturation 0 NoSaturation, 1 SaturateFinite,
 *        nearest-even whatever `rounding` (__nv_cvt_float_to_fp8);
 *   4 f16, 5 bf16, 8 e4m3, 9 e5m2 -> 6 f32: exact;
 *   any type to itself (1..9): a copy.
 * The codes equal the reference's lowering (CudaCodegen.scala:405-449,506-538)
 * bit for bit.  Other pairs return F4S_STATUS_INVALID_ARGUMENT with the
 * reference's message ("cannot emit a conversion from float to double").
 * Buffers aligned to their element sizes (32-byte alignment of both takes
 * the vector path).  One launch; asynchronous on `stream`. */
int f4s_convert(f4s_hotpath* hotpath, uint64_t stream, int32_t from_type, int32_t to_type, int32_t rounding,
                int32_t saturation, uint64_t in, uint64_t out, uint64_t n);

/* ------------------------------------------------------------ block sum */

/* The reference's blockReduceSum
 * (runtime/src/test/scala/flight4s/runtime/cuda/CudaResourcesJniSuite.scala:229-312)
 * extended to n elements: partials[t] = fp32 tree sum of tile t (256
 * elements, zero padded, the reference's stride order 128..1), then the same
 * tree over runs of 256 partials until one value remains in out[0].
 * Bit-identical to the reference kernel applied level by level.
 * Asynchronous on `stream`: up to 2^23 elements two launches (the tile
 * pass, then a one-CTA pass over the partials launched as its programmatic
 * dependent; the workspace is not touched), above that one clustered launch
 * that keeps a ticket and per-cluster partials in the workspace (zeroed once
 * by the caller; the kernel leaves it zeroed).  Calls sharing a workspace
 * must not overlap on the GPU. */
uint64_t f4s_block_reduce_workspace_bytes(int32_t n);
int f4s_block_reduce_sum_f32(f4s_hotpath* hotpath, uint64_t stream, uint64_t in, int32_t n, uint64_t partials,
                             uint64_t out, uint64_t workspace, uint64_t workspace_bytes);

/* Allocation-free form of f4s_block_reduce_sum_f32, for callers that cannot
 * allocate device memory (a host whose device memory belongs to another
 * allocator, code running where allocation is not allowed, callers with no
 * way to keep a workspace).  No counterpart in the reference.  The
 * workspace is a 64 KiB static device array in each CUDA context that loads
 * the library's device code (a GPU's primary context holds it until the
 * process exits); n must be <= 1,069,547,520 (else
 * F4S_STATUS_INVALID_ARGUMENT).  The first call in a context finds the
 * array's device address there and caches it under the context's id; that
 * call is rejected (F4S_STATUS_INVALID_ARGUMENT) while `stream` is being
 * captured, so make it before any capture.  All calls in a context share
 * the array: calls that overlap on the GPU race.  Never allocates. */
int f4s_block_reduce_sum_f32_noalloc(f4s_hotpath* hotpath, uint64_t stream, uint64_t in, int32_t n,
                                     uint64_t partials, uint64_t out);

/* ---------------------------------------------------------- elementwise */

/* The reference's vectorAdd (CudaResourcesJniSuite.scala:108-227; generated
 * text core/src/test/scala/flight4s/core/codegen/CudaCodegenSuite.scala:15-61):
 * output[i] = left[i] + right[i] for i < element_count.  The bf16 form
 * rounds the f32 sum to nearest-even. */
int f4s_vector_add_f32(f4s_hotpath* hotpath, uint64_t stream, uint64_t left, uint64_t right, uint64_t output,
                       int32_t element_count);
int f4s_vector_add_bf16(f4s_hotpath* hotpath, uint64_t stream, uint64_t left, uint64_t right, uint64_t output,
                        int32_t element_count);
/* The same `+` over every AdditiveType of the reference
 * (core/src/main/scala/flight4s/core/types/CudaType.scala:154-160) by
 * launch-ABI type code: 2 i32 and 3 u32 (32-bit wrap), 4 f16 and 5 bf16
 * (IEEE add rounded to nearest-even, the operation of `+` on __half /
 * __nv_bfloat16), 6 f32, 7 f64.  Other codes return
 * F4S_STATUS_INVALID_ARGUMENT. */
int f4s_vector_add(f4s_hotpath* hotpath, uint64_t stream, int32_t type_code, uint64_t left, uint64_t right,
                   uint64_t output, int32_t element_count);

/* ------------------------------------------------------------ row-wise */

/* bf16 [rows x cols] row-major, f32 math, bf16 round-to-nearest-even out:
 *   softmax: y = exp(x - max_row) / sum_row exp(x - max_row)
 *   rmsnorm: y = (x * rsqrt(mean_row(x^2) + eps)) * weight[col]        */
int f4s_softmax_rows_bf16(f4s_hotpath* hotpath, uint64_t stream, uint64_t in, uint64_t out, int32_t rows,
                          int32_t cols);
int f4s_rmsnorm_rows_bf16(f4s_hotpath* hotpath, uint64_t stream, uint64_t in, uint64_t weight, uint64_t out,
                          int32_t rows, int32_t cols, float eps);

/* ------------------------------------------------------------------ fp8 */

/* 1x128 block quantization of bf16 [rows x cols] to E4M3 with fused amax
 * (element conversion = the reference's convert.f32ToFP8E4M3, saturating,
 * round-to-nearest-even; core/src/main/scala/flight4s/core/codegen/CudaCodegen.scala:525-538):
 *   scales[r][b] = amax_b / 448, codes = e4m3(x * min(448 / amax_b, FLT_MAX))
 *   (0 when amax_b == 0); dequantize: y = bf16(f32(code) * scale).
 * codes: u8 [rows x cols]; scales: f32 [rows x ceil(cols / 128)]. */
int f4s_fp8_quantize_e4m3(f4s_hotpath* hotpath, uint64_t stream, uint64_t x, uint64_t codes, uint64_t scales,
                          int32_t rows, int32_t cols);
int f4s_fp8_dequantize_e4m3(f4s_hotpath* hotpath, uint64_t stream, uint64_t codes, uint64_t scales,
                            uint64_t y, int32_t rows, int32_t cols);

/* ---------------------------------------------------- synthetic inputs */

/* Philox4x32-10 synthetic data, elements [offset, offset + n) of the global
 * stream (so shards of one logical array can be generated per device).
 * kind: 0 uniform f32 [-1,1), 1 same as bf16, 2 normal f32 (p0 mean, p1 sd),
 * 3 normal bf16, 4 uniform i32 [ilo, ihi], 5 normal bf16 with outliers
 * (probability p2, factor p3). */
int f4s_fill_synthetic(f4s_hotpath* hotpath, uint64_t stream, uint64_t out, uint64_t n, uint64_t offset,
                       uint64_t seed, uint32_t stream_id, int32_t kind, float p0, float p1, float p2, float p3,
                       int32_t ilo, int32_t ihi);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* FLIGHT4S_B200_H_ */
