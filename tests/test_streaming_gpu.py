"""flash_attn_func_host: pinned host tensors streamed through the GPU in batch
chunks.  It runs the same kernel as flash_attn_func, so its host results must
equal the device call's bit for bit, for every chunking."""
import pytest
import torch

from oracle.attention_oracle import make_inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize(
    "b,s,h,hk,d,dtype,causal,chunks",
    [
        (5, 300, 4, 4, 128, torch.bfloat16, True, 2),  # uneven chunks (3 + 2)
        (3, 512, 2, 2, 64, torch.float16, False, 16),  # more chunks than batch entries
        (7, 256, 8, 2, 128, torch.bfloat16, False, 3),  # GQA, ring slots reused
        (1, 1000, 2, 1, 64, torch.float16, True, 4),
    ],
)
def test_host_streaming_matches_device_call(b, s, h, hk, d, dtype, causal, chunks):
    from flash_attention import flash_attn_func, flash_attn_func_host

    q, k, v = make_inputs(b, s, h, d, dtype, seed=37, heads_k=hk)
    o_dev, lse_dev = flash_attn_func(q.cuda(), k.cuda(), v.cuda(), causal, return_lse=True)
    qh, kh, vh = (t.pin_memory() for t in (q, k, v))
    o_h, lse_h = flash_attn_func_host(qh, kh, vh, causal, return_lse=True, chunks=chunks)
    assert not o_h.is_cuda and o_h.is_pinned()
    assert torch.equal(o_h, o_dev.cpu()) and torch.equal(lse_h, lse_dev.cpu())
    # caller-provided output buffers, O only
    out = torch.full_like(qh, 3.0).pin_memory()
    r = flash_attn_func_host(qh, kh, vh, causal, out=out, chunks=chunks)
    assert r is out and torch.equal(out, o_dev.cpu())


def test_host_streaming_rejects_device_tensors():
    from flash_attention import flash_attn_func_host

    x = torch.zeros(1, 8, 2, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="must be a CPU tensor"):
        flash_attn_func_host(x, x, x)
