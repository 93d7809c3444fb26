"""Failure path of the kernels' bounded waits, without faulting the GPU: a
one-CTA self-test kernel waits on a barrier phase that nothing completes;
the wait gives up after its limit, records NSA_ERR_TIMEOUT in the device
error word (read and cleared by device_error) and returns, and the context
still runs a correct decode afterwards."""
import importlib

import pytest
import torch

from oracle import attention as oa

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
pkg = importlib.import_module("numerics-and-sparse-attn_b200")
_lib = pkg._lib


def test_bounded_wait_reports_timeout_and_context_survives():
    assert pkg.device_error(DEV) == _lib.NSA_OK
    stream = torch.cuda.current_stream(DEV).cuda_stream
    _lib.check(_lib.load().nsa_selftest_wait_timeout(50_000_000, stream))  # 50 ms limit
    assert pkg.device_error(DEV) == _lib.NSA_ERR_TIMEOUT
    assert pkg.device_error(DEV) == _lib.NSA_OK  # reading cleared it
    g = torch.Generator().manual_seed(1)
    q = torch.randn(2, 64, 128, generator=g).half()
    k = torch.randn(2, 8, 100, 128, generator=g).half()
    v = torch.randn(2, 8, 100, 128, generator=g).half()
    o = pkg.dense_decode_attention(q.to(DEV), k.to(DEV), v.to(DEV), seq_len=100)
    ref = oa.dense_attention(q.float(), k.float(), v.float())
    assert (o.float().cpu() - ref).abs().max().item() < 2e-3
    assert pkg.device_error(DEV) == _lib.NSA_OK


def test_selftest_rejects_unbounded_limits():
    stream = torch.cuda.current_stream(DEV).cuda_stream
    for bad in (0, -1, 3_000_000_000):
        with pytest.raises(ValueError):
            _lib.check(_lib.load().nsa_selftest_wait_timeout(bad, stream))
