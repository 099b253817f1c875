"""torch.ops.b200ar: schemas, Meta implementations and torch.compile tracing
without graph breaks (CPU only: meta tensors, no kernel runs)."""

import pytest
import torch
import torch.distributed as dist

from dist_util import free_port


def _meta(*shape):
    return torch.empty(*shape, device="meta", dtype=torch.bfloat16)


def test_schemas_mark_outputs_as_mutated():
    import b200ar  # noqa: F401 - registers the operators

    ops = torch.ops.b200ar
    assert "Tensor(a!) out" in str(ops.all_reduce.default._schema)
    s = str(ops.all_reduce_residual_rmsnorm.default._schema)
    assert "Tensor(a!) y" in s and "Tensor(b!) residual_out" in s
    assert "Tensor(a!) y" in str(ops.rmsnorm.default._schema)
    assert "Tensor(a!) y" in str(ops.silu_mul.default._schema)


def test_meta_implementations_check_shapes():
    import b200ar  # noqa: F401

    torch.ops.b200ar.all_reduce(1, _meta(8, 64), _meta(8, 64))
    torch.ops.b200ar.rmsnorm(_meta(8, 64), _meta(64), 1e-5, _meta(8, 64))
    torch.ops.b200ar.silu_mul(_meta(8, 128), _meta(8, 64))
    torch.ops.b200ar.all_reduce_residual_rmsnorm(1, _meta(8, 64), _meta(8, 64), _meta(64), 1e-5, _meta(8, 64),
                                                 _meta(8, 64))
    with pytest.raises(RuntimeError, match="mismatch"):
        torch.ops.b200ar.all_reduce(1, _meta(8, 64), _meta(8, 32))
    with pytest.raises(RuntimeError, match="shape mismatch"):
        torch.ops.b200ar.silu_mul(_meta(8, 128), _meta(8, 128))


@pytest.mark.parametrize("backend", ["eager", "aot_eager"])
def test_layer_ops_trace_without_graph_breaks(backend):
    from b200ar.ops.layers import rmsnorm, silu_mul

    def step(x, g):
        y = rmsnorm(x, g, 1e-5)
        return silu_mul(torch.cat([y, y], dim=1)) * 2

    torch._dynamo.reset()
    out = torch.compile(step, fullgraph=True, backend=backend)(_meta(4, 64), _meta(64))
    assert out.shape == (4, 64) and out.device.type == "meta"


class _NativeStandIn:
    """Stands in for the CUDA communicator object: the traced branch only
    needs `_comm is not None` and the integer handle."""


def test_custom_allreduce_traces_to_dispatcher_ops():
    from b200ar import CustomAllreduce

    owns = not dist.is_initialized()
    if owns:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{free_port()}", rank=0, world_size=1)
    comm = CustomAllreduce(device="cpu", max_size=1 << 20)
    real = comm._comm
    comm._comm, comm._handle = _NativeStandIn(), 12345
    try:
        def layer(x, res, g):
            s = comm.all_reduce(x)
            y, z = comm.all_reduce_residual_rmsnorm(s, res, g, 1e-5)
            return y + z

        torch._dynamo.reset()
        out = torch.compile(layer, fullgraph=True, backend="aot_eager")(_meta(8, 64), _meta(8, 64), _meta(64))
        assert out.shape == (8, 64)
        assert comm.handle == 12345
    finally:
        comm._comm = real
        comm.close()
        if owns:
            dist.destroy_process_group()
