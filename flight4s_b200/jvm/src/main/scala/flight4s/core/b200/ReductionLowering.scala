// Not compiled here: this image has no JDK, Scala or sbt.  Written against
// the reference's IR (core/src/main/scala/flight4s/core/ir/IR.scala) for a
// maintainer to add to its core module; the tests beside it follow the style
// of core/src/test/scala/flight4s/core/ir/ReductionSuite.scala.
package flight4s.core.b200

import flight4s.core.ir.*
import flight4s.core.types.*

/** What the B200 kernels need to take over one `ReduceSum`: the global buffer
  * it reads, the launch-ABI code of the element type (which picks the kernel,
  * `f4s_reduce_sum_policy`), the policy ordinal and the range and initial
  * value expressions, which the host evaluates before the launch.
  */
final case class ReductionPlan(
    bufferName: String,
    inputTypeCode: Byte,
    policyOrdinal: Int,
    from: Expr[Int],
    until: Expr[Int],
    initial: Expr[?]
)

/** A kernel whose whole effect is `out(0) = reduceSum(i, from, until, init)(in(i))`
  * (optionally under `if (threadIdx.x == 0)`): the B200 path replaces the
  * launch of the generated serial loop by one `f4s_reduce_sum_policy` call and
  * a store of its result.
  */
final case class KernelReductionPlan(reduction: ReductionPlan, outputName: String)

object ReductionLowering:

  /** Launch-ABI descriptor code of an `AccumulatorType` input
    * (core/src/main/scala/flight4s/core/abi/CudaAbi.scala:12-21); the kernels
    * exist for exactly the reference's accumulator inputs
    * (core/src/main/scala/flight4s/core/types/CudaType.scala:199-230).
    */
  def inputTypeCode(valueType: CudaType[?]): Option[Byte] =
    valueType match
      case I32 => Some(2)
      case U32 => Some(3)
      case F16 => Some(4)
      case BF16 => Some(5)
      case F32 => Some(6)
      case F64 => Some(7)
      case FP8E4M3 => Some(8)
      case FP8E5M2 => Some(9)
      case _ => None

  /** ReductionPolicy (ir/IR.scala:79-82) as the C ABI's policy argument:
    * Strict 0, Deterministic 1 (both the order-fixed kernels), Fast 2.
    */
  def policyOrdinal(policy: ReductionPolicy): Int =
    policy match
      case ReductionPolicy.Strict => 0
      case ReductionPolicy.Deterministic => 1
      case ReductionPolicy.Fast => 2

  /** The plan for `reduction` when its value is a plain read of one global
    * buffer at the reduction index (`in(i)`), the form the kernels compute;
    * None for anything else (a transformed value, a shared or local array,
    * an index expression other than the reduction index), which keeps the
    * reference's serial lowering (codegen/CudaCodegen.scala:383-403).
    */
  def plan(reduction: ReduceSum[?, ?]): Option[ReductionPlan] =
    readOfIndex(reduction.value, reduction.index).flatMap { case (buffer, valueType) =>
      inputTypeCode(valueType).map { code =>
        ReductionPlan(buffer, code, policyOrdinal(reduction.policy), reduction.from, reduction.until,
          reduction.initial)
      }
    }

  private def readOfIndex(value: Expr[?], index: ReductionIndex): Option[(String, CudaType[?])] =
    value match
      case Load(element: BufferElement[?, ?], _) if isIndex(element.index, index) =>
        Some(element.bufferName -> element.valueType)
      case ToAccumulator(inner, _, _) => readOfIndex(inner, index)
      case _ => None

  private def isIndex(expr: Expr[Int], index: ReductionIndex): Boolean =
    expr match
      case ReductionIndex(name, _) => name == index.name
      case _ => false

  /** The kernel-level pattern: the body stores one reduction into element 0
    * of an output buffer, directly or under a `threadIdx.x == 0` guard.
    */
  def planKernel(body: Block): Option[KernelReductionPlan] =
    body.statements match
      case Vector(store: Store[?, ?]) => storeOfReduction(store)
      case Vector(IfThen(Compare(ComparisonOperator.Equal, Intrinsic("threadIdx.x", _, _), Literal(0, _, _), _, _),
            Block(Vector(store: Store[?, ?])), None, _)) =>
        storeOfReduction(store)
      case _ => None

  private def storeOfReduction(store: Store[?, ?]): Option[KernelReductionPlan] =
    (store.to, store.value) match
      case (out: BufferElement[?, ?], reduction: ReduceSum[?, ?]) if isZero(out.index) =>
        plan(reduction).map(KernelReductionPlan(_, out.bufferName))
      case _ => None

  private def isZero(expr: Expr[Int]): Boolean =
    expr match
      case Literal(0, _, _) => true
      case _ => false
