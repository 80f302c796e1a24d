"""Host-side checks of the drop-in operators (ryzenai-npu-lab_b200/operators.py),
which raise ValueError like the reference's operators do for an out-of-range
length (experiments/lfm25_attention_context_cache_kernel.py:25-26,
experiments/lfm25_attention_chunked_cache_kernel.py:25-26) before any work
is queued; no GPU is needed for these."""
import pytest
import torch

from conftest import load_pkg

BF = torch.bfloat16


def test_out_of_range_lengths_raise_value_error():
    ops = load_pkg("operators")
    t = torch.zeros(8, dtype=BF)
    with pytest.raises(ValueError, match="past_length"):
        ops.attention_context_cache(t, t, t, t, past_length=0)
    with pytest.raises(ValueError, match="block_count"):
        ops.attention_context_chunked(t, t, t, t, block_count=0)


def test_buffers_must_be_cuda_bf16_of_the_right_size():
    ops = load_pkg("operators")
    cpu = torch.zeros(3072, dtype=BF)
    with pytest.raises(ValueError, match="CUDA bfloat16"):
        ops.attention_context_cache(cpu, torch.zeros(8 * 2 * 21 * 64, dtype=BF), torch.zeros(2048, dtype=BF),
                                    torch.zeros(8 * 2 * 22 * 64, dtype=BF), past_length=21)
    with pytest.raises(ValueError, match="CUDA bfloat16"):
        ops.attention_context_cache(cpu.float(), cpu, cpu, cpu, past_length=21)
    with pytest.raises(ValueError):
        ops.append_attention_cache(torch.zeros(100, dtype=BF), cpu, cpu)
