"""Guard regions around the symmetric buffers of the fused collectives (CPU).

The allocation helper is exercised with a stand-in for torch's symmetric
memory module that returns ordinary host tensors: the data view must sit
between two 4 KiB guards holding the pattern, and a write one element past
either end of the data must be counted."""
import torch

from bloom_b200.parallel import fused


class _HostSymm:
    @staticmethod
    def empty(n, dtype, device):
        return torch.zeros(n, dtype=dtype)


def test_guards_surround_the_data():
    for dtype in (torch.bfloat16, torch.int32):
        full, data, g = fused._guarded(_HostSymm, 1000, dtype, "cpu")
        es = full.element_size()
        assert g * es == fused.CANARY_BYTES and data.numel() == 1000
        assert data.data_ptr() - full.data_ptr() == fused.CANARY_BYTES
        assert fused._bad_guard_words(full) == 0
        data.fill_(7)  # writes inside the data never touch the guards
        assert fused._bad_guard_words(full) == 0
        full[g + 1000] = 1  # one element past the end
        full[g - 1] = 1  # one element before the start
        assert fused._bad_guard_words(full) == 2


def test_guard_pattern_is_finite_bf16():
    w = torch.tensor([fused.CANARY_WORD], dtype=torch.int64).to(torch.int32)
    assert torch.isfinite(w.view(torch.bfloat16).float()).all()
