// Not compiled here: this image has no JDK, Scala or sbt.  Written for the
// reference's runtime package (runtime/src/main/scala/flight4s/runtime/cuda/)
// so it can reach the package-private native handles; it needs one accessor
// added to CudaDeviceBuffer (runtime/src/main/scala/flight4s/runtime/cuda/CudaResources.scala:861-867):
//     private[cuda] def nativeAddress: Long = handle
// and the timing event mode of CudaEvent (CudaResources.scala:104-106):
//     case Timing extends CudaEventMode(0)   // CU_EVENT_DEFAULT: timing enabled
package flight4s.runtime.cuda

import flight4s.core.b200.{ReductionLowering, ReductionPlan}
import flight4s.core.ir.ReductionPolicy
import flight4s.core.types.CudaType
import flight4s.runtime.cuda.b200.B200NativeBindings

/** The sm_100a hot path of one context: the embedded module loaded once,
  * reductions launched through it on the context's streams.  Results come
  * back the way the reference's serial ReduceSum would deliver them to a
  * caller: an f64 for the floating-point inputs (F32 sums carried in f64,
  * whose f32 rounding is the correctly rounded sum), the 32-bit wrap for
  * I32 / U32.
  */
final class B200Reductions private (val context: CudaContext, private val hotpath: Long) extends AutoCloseable:

  /** ReduceSum of `buffer(from until until)`, any accumulator input type,
    * under `policy`.  Blocks until the result is on the host (the
    * reference's serial loop returns a value too).
    */
  def reduceSum[T](
      buffer: CudaDeviceBuffer[T],
      from: Long,
      until: Long,
      policy: ReductionPolicy,
      stream: CudaStream
  ): Either[CudaDriverFailure, Double] =
    require(0 <= from && from <= until && until <= buffer.elementCount, s"range [$from, $until) outside the buffer")
    val code = ReductionLowering.inputTypeCode(buffer.valueType).getOrElse(
      throw IllegalArgumentException(s"no ReduceSum accumulator for ${buffer.valueType.cudaName}"))
    val ordinal = ReductionLowering.policyOrdinal(policy)
    val n = until - from
    val wsBytes = B200NativeBindings.reducePolicyWorkspaceBytes(hotpath, code, ordinal, n)
    if wsBytes < 0 then Left(lastFailure("sizing the reduction workspace"))
    else
      // the workspace as 4-byte words, the result as one 8-byte slot (f64
      // bits, or the 32-bit wrap in its low word): the reference's CudaTypes
      // have no byte or 64-bit integer buffer type
      for
        ws <- context.allocate[Int](math.max((wsBytes + 3) / 4, 1L).toInt)(using flight4s.core.types.I32)
        out <- context.allocate[Double](1)(using flight4s.core.types.F64)
        _ <- status(
          B200NativeBindings.reduceSumPolicy(hotpath, stream.nativeHandle, code, ordinal,
            buffer.nativeAddress + from * buffer.valueType.sizeBytes, n, out.nativeAddress, ws.nativeAddress,
            4L * ws.elementCount, false),
          "ReduceSum launch")
        _ <- stream.synchronize()
        value <- out.copyToArray().map(_.head)
      yield
        ws.close(); out.close()
        if code == 2 || code == 3 then java.lang.Double.doubleToRawLongBits(value).toInt.toDouble else value

  /** Run a planned reduction (ReductionLowering.plan) whose range and initial
    * value the caller has evaluated.
    */
  def run[T](plan: ReductionPlan, buffer: CudaDeviceBuffer[T], from: Long, until: Long, initial: Double,
             stream: CudaStream): Either[CudaDriverFailure, Double] =
    val policy = ReductionPolicy.fromOrdinal(plan.policyOrdinal)
    reduceSum(buffer, from, until, policy, stream).map(initial + _)

  override def close(): Unit =
    B200NativeBindings.hotpathClose(hotpath)

  private def status(code: Int, what: String): Either[CudaDriverFailure, Unit] =
    if code == 0 then Right(()) else Left(lastFailure(what))

  private def lastFailure(what: String): CudaDriverFailure = B200Reductions.lastFailure(what)

object B200Reductions:
  def open(context: CudaContext): Either[CudaDriverFailure, B200Reductions] =
    val handle = B200NativeBindings.hotpathOpen(context.nativeHandle)
    if handle == 0L then Left(lastFailure("loading the sm_100a hot path"))
    else Right(new B200Reductions(context, handle))

  private def lastFailure(what: String): CudaDriverFailure =
    CudaDriverFailure(what, B200NativeBindings.lastStatusCode(), "", B200NativeBindings.lastStatusDescription(), "", "")

  /** Elapsed milliseconds between two events created with the timing mode. */
  def elapsedMillis(start: CudaEvent, end: CudaEvent): Float =
    require(start.context eq end.context, "events of different contexts")
    B200NativeBindings.eventElapsedMs(start.context.nativeHandle, start.nativeHandle, end.nativeHandle)
