"""Host-tier arena allocation policy (CPU only, no device calls): registration is retried
on a fresh range and falls back to the pinned allocator, as the decode stacks rely on
when another process has just released its own page-locked arena."""
import torch

from tideway_b200.stack import alloc_host_arena


def test_register_retries_on_a_fresh_range():
    seen = []

    def register(ptr, nbytes):
        seen.append((ptr, nbytes))
        if len(seen) < 3:
            raise RuntimeError("cudaHostRegister failed: OS call failed")

    arena, registered = alloc_host_arena(1024, register=register, retry_s=30.0, pause_s=0.0)
    assert registered and arena.numel() == 1024 and arena.dtype == torch.bfloat16
    assert len(seen) == 3 and all(n == 2048 for _, n in seen)


def test_falls_back_to_the_pinned_allocator():
    calls = []

    def register(ptr, nbytes):
        calls.append(nbytes)
        raise RuntimeError("cudaHostRegister failed: OS call failed")

    fallback = []

    def pinned_alloc(n):
        fallback.append(n)
        return torch.zeros(n, dtype=torch.bfloat16)

    arena, registered = alloc_host_arena(512, register=register, pinned_alloc=pinned_alloc,
                                         retry_s=0.0, pause_s=0.0)
    assert not registered and fallback == [512] and arena.numel() == 512 and len(calls) >= 1
