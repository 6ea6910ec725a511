"""Per-rank partials from the oracle for the CPU (gloo) tests of the sharded
reducer: stands in for the hot path, writing each shard's partial into the
reducer's partial tensor the way the kernels write it."""
import numpy as np


class OraclePartials:
    workspace_bytes = 0

    def reduce_into(self, op, shard, out, n, stream, index_base, workspace):
        import flight4s_b200 as f4s
        from oracle import oracle as orc
        x = np.ascontiguousarray(shard.numpy()[:n])
        if op == f4s.REDUCE_SUM_F32:
            out[0] = orc.sum_f32_exact(x)[0]
        elif op == f4s.REDUCE_SUM_I32:
            out[0] = int(orc.sum_i32(x))
        elif op == f4s.REDUCE_ARGMAX_F32:
            v, i = orc.argmax_f32(x)
            out[0] = orc.argmax_packed_key(v, i + index_base) if i >= 0 else -(1 << 63)
            out[1] = i + index_base if i >= 0 else -1
        else:
            raise ValueError(op)
