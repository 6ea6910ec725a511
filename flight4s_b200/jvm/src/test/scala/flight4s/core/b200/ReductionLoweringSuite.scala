// Not compiled here: this image has no JDK, Scala or sbt.  munit cases in the
// style of the reference's core/src/test/scala/flight4s/core/ir/ReductionSuite.scala.
package flight4s.core.b200

import munit.FunSuite

import flight4s.core.dsl.CudaDsl.*
import flight4s.core.ir.*
import flight4s.core.types.*

class ReductionLoweringSuite extends FunSuite:

  test("a plain read of a global buffer at the reduction index is planned"):
    val definition = kernel("sum", params(input[Float]("in"), output[Float]("out"), value[Int]("n"))) {
      case (in, out, n) =>
        out(literal(0)) := reduceSum("i", literal(0), n, literal(0.0f), ReductionPolicy.Deterministic)(i => in(i))
    }
    val reduction = definition.body.statements.collectFirst { case Store(_, r: ReduceSum[?, ?], _) => r }.get
    val plan = ReductionLowering.plan(reduction).get
    assertEquals(plan.bufferName, "in")
    assertEquals(plan.inputTypeCode, 6.toByte)
    assertEquals(plan.policyOrdinal, 1)
    assertEquals(ReductionLowering.planKernel(definition.body).map(_.outputName), Some("out"))

  test("every accumulator input type maps to its launch-ABI code"):
    assertEquals(
      Vector(I32, U32, F16, BF16, F32, F64, FP8E4M3, FP8E5M2).map(ReductionLowering.inputTypeCode),
      Vector[Option[Byte]](Some(2), Some(3), Some(4), Some(5), Some(6), Some(7), Some(8), Some(9))
    )

  test("policies map to the C ABI's ordinals"):
    assertEquals(
      Vector(ReductionPolicy.Strict, ReductionPolicy.Deterministic, ReductionPolicy.Fast)
        .map(ReductionLowering.policyOrdinal),
      Vector(0, 1, 2)
    )

  test("a transformed value keeps the serial lowering"):
    val reduction = reduceSum("i", literal(0), literal(8), literal(0.0f))(_ => literal(1.0f))
      .asInstanceOf[ReduceSum[Float, Float]]
    assertEquals(ReductionLowering.plan(reduction), None)
