"""When the fused NVLink collectives are chosen, checked on CPU with the
process group and the GPU inventory faked.

The fused kernels wait on their peers inside the kernel, so every rank must
own its own GPU: two ranks on one GPU (gloo, or a device override that puts
two NCCL ranks on the same GPU) must get the library collectives instead.
"""

import torch

from minispeed_b200.parallel import fused


def _fake_group(monkeypatch, backend, identities, world=2):
    monkeypatch.setattr(fused.comm, "is_distributed", lambda: True)
    monkeypatch.setattr(fused.comm, "get_world_size", lambda: world)
    monkeypatch.setattr(torch.distributed, "get_backend", lambda *a, **k: backend)
    monkeypatch.setattr(fused, "_device_identity", lambda device: "unused")
    monkeypatch.setattr(fused.comm, "all_gather_object", lambda obj: list(identities))
    monkeypatch.delenv("LOCAL_WORLD_SIZE", raising=False)


def test_shared_gpu():
    assert fused.shared_gpu(["h/GPU-a", "h/GPU-a"])
    assert not fused.shared_gpu(["h/GPU-a", "h/GPU-b"])
    assert not fused.shared_gpu(iter(["h/GPU-a", "h/GPU-b"]))


def test_cpu_device_is_refused():
    ok, why = fused.supported(torch.device("cpu"))
    assert not ok and "CUDA" in why


def test_gloo_group_is_refused(monkeypatch):
    _fake_group(monkeypatch, "gloo", ["h/0", "h/1"])
    ok, why = fused.supported(torch.device("cuda", 0))
    assert not ok and "gloo" in why


def test_two_nccl_ranks_on_one_gpu_are_refused(monkeypatch):
    _fake_group(monkeypatch, "nccl", ["h/GPU-a", "h/GPU-a"])
    ok, why = fused.supported(torch.device("cuda", 0))
    assert not ok and "same GPU" in why


def test_ranks_across_nodes_are_refused(monkeypatch):
    _fake_group(monkeypatch, "nccl", ["a/0", "b/0"])
    monkeypatch.setenv("LOCAL_WORLD_SIZE", "1")
    ok, why = fused.supported(torch.device("cuda", 0))
    assert not ok and "node" in why


def test_device_identity_uses_uuid_bytes(monkeypatch):
    class Uuid:
        bytes = list(range(16))

    class Props:
        uuid = Uuid()

    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda d: Props())
    a = fused._device_identity(torch.device("cuda", 0))
    b = fused._device_identity(torch.device("cuda", 5))
    assert a == b and a.endswith("/000102030405060708090a0b0c0d0e0f")   # same GPU, any index

    class NoUuid:
        pass

    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda d: NoUuid())
    assert fused._device_identity(torch.device("cuda", 5)).endswith("/index5")
