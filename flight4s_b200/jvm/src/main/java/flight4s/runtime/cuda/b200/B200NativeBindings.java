// Not compiled here: this image has no JDK.  JNI declarations of the
// libflight4s_b200.so entry points the Scala side below calls; each one is a
// thin forward to the C function of the same meaning in
// include/flight4s_b200.h (stubs in INTEGRATION.md section 1).  Handles are
// the same jlong values the reference's CudaNativeBindings passes
// (runtime/src/main/java/flight4s/runtime/cuda/internal/CudaNativeBindings.java).
package flight4s.runtime.cuda.b200;

public final class B200NativeBindings {
  static {
    String path = System.getProperty("flight4s.b200.native.path");
    if (path != null) System.load(path); else System.loadLibrary("flight4s_b200_jni");
  }

  private B200NativeBindings() {}

  /** f4s_hotpath_open: loads the sm_100a module into the context; returns the hot-path handle. */
  public static native long hotpathOpen(long context);

  /** f4s_hotpath_close. */
  public static native int hotpathClose(long hotpath);

  /** f4s_hotpath_set_launch_overlap (0 or 1). */
  public static native int setLaunchOverlap(long hotpath, int enable);

  /** f4s_reduce_policy_workspace_bytes: workspace bytes for (type code, policy, n), or -1. */
  public static native long reducePolicyWorkspaceBytes(long hotpath, byte inputType, int policy, long n);

  /**
   * f4s_reduce_sum_policy: ReduceSum of n elements at device address `in` of launch-ABI type
   * `inputType` under ReductionPolicy ordinal `policy` (Strict 0, Deterministic 1, Fast 2);
   * the result (f64 bits, or the 32-bit wrap for I32/U32) lands at device address `out`.
   */
  public static native int reduceSumPolicy(long hotpath, long stream, byte inputType, int policy, long in, long n,
                                           long out, long workspace, long workspaceBytes, boolean accumulate);

  /** f4s_reduce_argmax: 16-byte record {packed or 64-bit key, index} at `out`. */
  public static native int reduceArgmax(long hotpath, long stream, byte inputType, long in, long n, long out,
                                        long workspace, long workspaceBytes, long indexBase, boolean accumulate);

  /** f4s_event_elapsed_ms between two timing-enabled events; NaN on failure. */
  public static native float eventElapsedMs(long context, long startEvent, long endEvent);

  /** Status of the calling thread's last call: code, name, description (f4s_last_status_*). */
  public static native int lastStatusCode();

  public static native String lastStatusDescription();
}
