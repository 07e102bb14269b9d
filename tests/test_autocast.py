"""autocast / autocast_dtype / float32_function against the reference's rules
(namitorch/amp.py:18-75), the ``linear`` consumer of the autocast policy
(namitorch/nn/functional.py:44-65), and the out-of-memory error of the flat arenas
(namitorch/backends/_cuda_memory.py:8-21).

Deliberate difference: autocast also accepts bfloat16 (the reference takes float16 only).
"""
import pytest
import torch

from namitorch_b200 import amp
from namitorch_b200.errors import NamiTorchCUDAOutOfMemoryError
from namitorch_b200.nn import functional as F


def _state():
    return amp._autocast_state.get()


def test_autocast_argument_errors():
    with pytest.raises(ValueError, match="device_type must be 'cuda' or 'cpu'"):
        with amp.autocast("tpu"):
            pass
    with pytest.raises(TypeError, match="enabled must be a Python bool"):
        with amp.autocast("cuda", enabled=1):
            pass
    with pytest.raises(ValueError, match="float16 and bfloat16"):
        with amp.autocast("cuda", dtype=torch.float32):
            pass
    with pytest.raises(RuntimeError, match="CPU autocast is not supported"):
        with amp.autocast("cpu"):
            pass


def test_disabled_cpu_autocast_is_a_no_op():
    before = _state()
    with amp.autocast("cpu", enabled=False):
        assert _state() == before
    assert _state() == before


def test_nesting_restores_the_outer_state_also_after_exceptions():
    assert _state() == (False, torch.float16)
    with amp.autocast("cuda", dtype=torch.bfloat16):
        assert _state() == (True, torch.bfloat16)
        with amp.autocast("cuda", enabled=False):
            assert _state() == (False, torch.float16)
            with amp.autocast("cuda", dtype="float16"):
                assert _state() == (True, torch.float16)
            assert _state() == (False, torch.float16)
        assert _state() == (True, torch.bfloat16)
        with pytest.raises(KeyError):
            with amp.autocast("cuda"):
                raise KeyError("inside")
        assert _state() == (True, torch.bfloat16)
    assert _state() == (False, torch.float16)


def test_autocast_dtype_is_none_outside_the_float16_policy_or_off_the_gpu():
    x = torch.ones(2, 3)
    with amp.autocast("cuda"):
        assert amp.autocast_dtype("linear", x) is None             # CPU operands are left alone
        assert amp.autocast_dtype("softmax", x) is None            # float32 policy
        assert amp.autocast_dtype("linear") is None                # no operands
        assert amp.autocast_dtype("linear", None, None) is None
    assert amp.autocast_dtype("matmul", x) is None                 # autocast off


def test_policy_table_matches_the_reference():
    low = sorted(k for k, v in amp.OPERATION_POLICIES.items() if v == "low")
    assert low == ["linear", "matmul"]
    for name in ("softmax", "log_softmax", "cross_entropy", "layer_norm", "rms_norm", "sum", "exp", "gelu"):
        assert amp.OPERATION_POLICIES[name] == "float32"


def test_float32_function_promotes_low_precision_arguments():
    def softmax(x, *, other=None):
        return x.dtype, None if other is None else other.dtype

    wrapped = amp.float32_function(softmax)
    assert wrapped.__name__ == "softmax"
    assert wrapped(torch.ones(2, dtype=torch.float16), other=torch.ones(1, dtype=torch.bfloat16)) == \
        (torch.float32, torch.float32)
    assert wrapped(torch.ones(2, dtype=torch.float64)) == (torch.float64, None)

    def matmul(x):
        return x

    with pytest.raises(ValueError, match="No float32 policy for matmul"):
        amp.float32_function(matmul)


def test_linear_checks_like_the_reference():
    w = torch.ones(4, 3)
    with pytest.raises(TypeError, match="input and weight must be"):
        F.linear([1.0], w)
    with pytest.raises(ValueError, match="weight must have rank 2"):
        F.linear(torch.ones(3), torch.ones(3))
    with pytest.raises(ValueError, match="last dimension 3"):
        F.linear(torch.ones(2, 5), w)
    with pytest.raises(ValueError, match=r"bias must have shape \(4,\)"):
        F.linear(torch.ones(2, 3), w, torch.ones(3))
    out = F.linear(torch.ones(2, 3), w, torch.zeros(4))
    assert torch.equal(out, torch.full((2, 4), 3.0))


def test_arena_out_of_memory_raises_the_reference_error(monkeypatch):
    """A failing arena allocation becomes NamiTorchCUDAOutOfMemoryError with the requested
    bytes (a host-side failure, faked here)."""
    from namitorch_b200 import flat

    def failing(*args, **kwargs):
        raise torch.OutOfMemoryError("CUDA out of memory (faked)")

    monkeypatch.setattr(flat.torch, "zeros", failing)
    with pytest.raises(NamiTorchCUDAOutOfMemoryError) as info:
        flat.zeroed_arena(1 << 20, torch.float32, "cpu")
    assert info.value.requested_bytes == 4 << 20
    assert "requested=4194304 bytes" in str(info.value)
    assert isinstance(info.value, MemoryError)


@pytest.mark.gpu
def test_autocast_dtype_and_linear_on_the_gpu(cuda_device):
    from namitorch_b200.optim import AdamW
    w = torch.nn.Parameter(torch.randn(64, 32, device=cuda_device) * 0.02)
    b = torch.nn.Parameter(torch.zeros(64, device=cuda_device))
    opt = AdamW([w, b], lr=1e-3, model_dtype=torch.bfloat16)   # w, b become views of the bf16 copy
    x = torch.randn(8, 32, device=cuda_device)
    with amp.autocast("cuda", dtype=torch.bfloat16):
        assert amp.autocast_dtype("linear", x, w) is torch.bfloat16
        assert amp.autocast_dtype("softmax", x) is None
        xs, ws, bs = amp.autocast_operands("linear", x, w, b)
        assert ws is w and bs is b                    # the persistent copy: no per-forward cast
        assert xs.dtype == torch.bfloat16 and xs is not x
        y = F.linear(x, w, b)
    assert y.dtype == torch.bfloat16
    ref = x @ opt.master_params[0].T + opt.master_params[1]
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2)
    # fp32 parameters are cast under autocast, and float16 stays the default dtype.
    w32 = torch.randn(64, 32, device=cuda_device)
    with amp.autocast("cuda"):
        _, w16 = amp.autocast_operands("matmul", x, w32)
        assert w16.dtype == torch.float16
        assert F.linear(x, w32).dtype == torch.float16


@pytest.mark.gpu
def test_arena_larger_than_the_device_raises_the_reference_error(cuda_device):
    """An arena request far beyond device memory (a host-side allocation failure)."""
    from namitorch_b200 import flat
    total = torch.cuda.mem_get_info(cuda_device)[1]
    with pytest.raises(NamiTorchCUDAOutOfMemoryError) as info:
        flat.zeroed_arena(4 * total, torch.float32, cuda_device)
    err = info.value
    assert err.requested_bytes == 16 * total
    assert err.total_bytes == total and err.free_bytes is not None and err.free_bytes <= total
    assert err.allocated_bytes is not None and err.reserved_bytes is not None
    torch.ones(1, device=cuda_device).sum().item()    # the device is still usable
