"""CPU checks of the Python binding's argument checks. The C ABI takes bare
device pointers with no lengths, so the binding refuses a wrong dtype, size
or layout before the call, the way Stage::wm refuses a width mismatch
(infer/mod.rs:139-145). No device is needed: the checks run before the
library is called, and a stand-in object plays the CUDA tensor."""
import numpy as np
import pytest
import torch

import ouroboros_b200 as oq
from ouroboros_b200 import _dev, _ptr, _rows


class FakeCuda:
    """Just enough of a CUDA tensor for the checks (nothing is dereferenced)."""

    def __init__(self, dtype, n, contiguous=True):
        self.dtype, self._n, self._c = dtype, n, contiguous
        self.is_cuda = True

    def is_contiguous(self):
        return self._c

    def numel(self):
        return self._n

    def data_ptr(self):
        return 0x1000


def _status(fn):
    with pytest.raises(oq.OuroqError) as e:
        fn()
    return e.value.status


def test_dev_accepts_the_exact_tensor():
    assert _dev(FakeCuda(torch.float32, 12), "float32", 12, "x") == 0x1000
    assert _dev(FakeCuda(torch.int64, 3), "int64", None, "pos") == 0x1000
    assert _dev(None, "float32", 12, "signs", optional=True) is None


def test_dev_refusals():
    assert _status(lambda: _dev(None, "float32", 4, "x")) == 7
    assert _status(lambda: _dev(torch.zeros(4), "float32", 4, "x")) == 7      # host tensor
    assert _status(lambda: _dev(np.zeros(4, np.float32), "float32", 4, "x")) == 7
    assert _status(lambda: _dev(FakeCuda(torch.float64, 4), "float32", 4, "x")) == 7
    assert _status(lambda: _dev(FakeCuda(torch.float32, 4, False), "float32", 4, "x")) == 7
    assert _status(lambda: _dev(FakeCuda(torch.float32, 5), "float32", 4, "x")) == 1
    assert _status(lambda: _dev(FakeCuda(torch.int64, 0), "int64", None, "pos")) == 1


def test_rows():
    assert _rows(torch.zeros(3, 8), 8, "x") == 3
    assert _rows(torch.zeros(8), 8, "x") == 1
    assert _rows(torch.zeros(0, 8), 8, "x") == 0
    assert _status(lambda: _rows(torch.zeros(2, 7), 8, "x")) == 1


def test_ptr_refuses_strided_buffers():
    assert _status(lambda: _ptr(torch.zeros(4, 4).t())) == 7
    assert _status(lambda: _ptr(np.zeros((4, 4), np.float32).T)) == 7
    assert _ptr(None) is None


def test_context_methods_check_before_calling_the_library():
    # a context object without a device: the library handle is never reached
    class NoLib:
        def __getattr__(self, name):
            return lambda *a: pytest.fail(f"{name} was called")

    ctx = oq.Context.__new__(oq.Context)
    ctx.lib, ctx.ctx = NoLib(), None
    w = oq.Weight(ctx, 0, oq.TERNARY2, 64, 256)
    x_cpu = torch.zeros(2, 256)
    assert _status(lambda: ctx.gemm_f32act(w, x_cpu, y=FakeCuda(torch.float32, 128))) == 7
    assert _status(lambda: ctx.gemm_f32act(w, torch.zeros(2, 100))) == 1  # width mismatch
    assert _status(lambda: ctx.gemm(w, torch.zeros(2, 200, dtype=torch.int8), None)) == 1
    x = FakeCuda(torch.float32, 2 * 256)
    x.shape = (2, 256)
    y_short = FakeCuda(torch.float32, 2 * 63)
    assert _status(lambda: ctx.gemm_f32act(w, x, y=y_short)) == 1
    assert _status(lambda: ctx.gemm_f32act_noalloc(w, x, FakeCuda(torch.float16, 128))) == 7
    assert _status(lambda: ctx.argmax_token(w, x, tokens=FakeCuda(torch.int32, 2))) == 7


def test_numpy_input_to_a_device_method_is_an_ouroq_error():
    class NoLib:
        def __getattr__(self, name):
            return lambda *a: pytest.fail(f"{name} was called")

    ctx = oq.Context.__new__(oq.Context)
    ctx.lib, ctx.ctx = NoLib(), None
    x = np.zeros((2, 256), np.float32)
    assert _status(lambda: ctx.quantize_act(x)) == 1
    assert _status(lambda: ctx.rotate(x)) == 1
    assert _status(lambda: ctx.quantize_group([x], [None], [None])) == 1
    w = oq.Weight(ctx, 0, oq.TERNARY2, 64, 256)
    assert _status(lambda: ctx.gemm_f32act(w, x)) == 7
    assert _status(lambda: ctx.argmax_token(w, x)) == 7
