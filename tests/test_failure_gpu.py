"""Failure paths of the device code, exercised without faulting the GPU.

* A peer-flag wait that nothing will satisfy (one process, one GPU: the "peer" slot of a
  flag array is simply never written) runs out of a short runtime wait budget, reports
  kErrPeerTimeout through the status word and returns; the context stays usable and the
  next kernel gives correct results.
* Out-of-range token ids and KV slot ids are caught by the kernels' bounds checks
  (kErrBadIndex with the offending index); the access is skipped, not performed.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _gemm_still_works(dev):
    from octopus_b200 import ops

    a = torch.randn(256, 512, device=dev).bfloat16()
    w = torch.randn(384, 512, device=dev).bfloat16()
    out = ops.gemm(a, w)
    ref = a.float() @ w.float().t()
    torch.cuda.synchronize(dev)
    ops.check_status(dev.index)
    assert float((out.float() - ref).norm() / ref.norm()) < 1e-2


def test_peer_barrier_times_out_and_context_survives():
    from octopus_b200 import ops

    dev = torch.device("cuda", 0)
    ops.check_status(0)
    flags = [torch.zeros(16, dtype=torch.int32, device=dev) for _ in range(2)]
    with ops.wait_budget(0, 1000):  # 1 ms
        ops.ext().peer_barrier([f.data_ptr() for f in flags], 0, 1, 0)
        torch.cuda.synchronize(dev)
    code, where, _ = ops.read_status(0)
    assert code == 2 and where == 901, (code, where)  # waited on slot 1, which no peer writes
    with pytest.raises(ops.KernelError) as e:
        ops.check_status(0)
    assert e.value.code == 2
    assert ops.read_status(0)[0] == 0  # cleared
    assert int(ops.ext().status_tensor(0)[2]) == 0  # budget restored to the default
    assert int(flags[0][0]) == 1 and int(flags[1][0]) == 1  # its own signal was delivered
    _gemm_still_works(dev)


def test_embedding_rejects_out_of_range_ids():
    from octopus_b200 import ops

    dev = torch.device("cuda", 0)
    ops.check_status(0)
    V, H = 1000, 256
    W = torch.randn(V, H, device=dev).bfloat16()
    ids = torch.tensor([3, 7, V + 5, 2], dtype=torch.int64, device=dev)
    out = ops.ext().embed_fwd(ids, W)
    torch.cuda.synchronize(dev)
    code, where, index = ops.read_status(0)
    assert (code, where, index) == (3, 700, V + 5)
    ops.read_status(0)
    with pytest.raises(ops.KernelError):
        ops.check_status(0)
    assert torch.equal(out[[0, 1, 3]], W[[3, 7, 2]])
    assert not out[2].any()  # the bad row was not read: zeros
    _gemm_still_works(dev)


def test_kv_write_rejects_out_of_range_slots():
    from octopus_b200 import ops

    dev = torch.device("cuda", 0)
    ops.check_status(0)
    Hq, Hkv, D, slots = 4, 2, 64, 32
    qkv = torch.randn(3, (Hq + 2 * Hkv) * D, device=dev).bfloat16()
    kc = torch.zeros(slots, Hkv * D, device=dev).bfloat16()
    vc = torch.zeros_like(kc)
    sl = torch.tensor([5, slots + 100, -1], dtype=torch.int64, device=dev)
    ops.ext().kv_write(qkv, Hq, Hkv, D, sl, kc, vc)
    torch.cuda.synchronize(dev)
    code, where, index = ops.read_status(0)
    assert (code, where, index) == (3, 710, slots + 100)
    with pytest.raises(ops.KernelError):
        ops.check_status(0)
    assert torch.equal(kc[5], qkv[0, Hq * D: (Hq + Hkv) * D])
    assert int((kc != 0).any(dim=1).sum()) == 1  # only the valid row was written
    _gemm_still_works(dev)
