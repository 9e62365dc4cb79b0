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
    o_h, lse_h = flash_attn_func_host(qh, kh, vh, causal, return_lse=True, chunks=chunks, min_chunk_bytes=0)
    assert not o_h.is_cuda and o_h.is_pinned()
    assert torch.equal(o_h, o_dev.cpu()) and torch.equal(lse_h, lse_dev.cpu())
    # caller-provided output buffers, O only
    out = torch.full_like(qh, 3.0).pin_memory()
    r = flash_attn_func_host(qh, kh, vh, causal, out=out, chunks=chunks, min_chunk_bytes=0)
    assert r is out and torch.equal(out, o_dev.cpu())
    # default chunk size: these small problems take the one-chunk path
    o_1, lse_1 = flash_attn_func_host(qh, kh, vh, causal, return_lse=True)
    assert torch.equal(o_1, o_dev.cpu()) and torch.equal(lse_1, lse_dev.cpu())


def test_host_streaming_workspace_follows_shapes():
    """The device ring kept between calls is re-made when shapes, dtype or
    chunk size change, and release_workspaces frees it."""
    from flash_attention import flash_attn_func, flash_attn_func_host
    from flash_attention.streaming import release_workspaces

    for b, s, h, hk, d, dtype in [(6, 256, 4, 4, 64, torch.float16), (6, 256, 4, 2, 64, torch.float16),
                                  (9, 384, 4, 4, 128, torch.bfloat16), (2, 128, 2, 2, 128, torch.bfloat16),
                                  (9, 384, 4, 4, 128, torch.bfloat16)]:
        q, k, v = make_inputs(b, s, h, d, dtype, seed=38 + b, heads_k=hk)
        want = flash_attn_func(q.cuda(), k.cuda(), v.cuda(), True).cpu()
        qh, kh, vh = (t.pin_memory() for t in (q, k, v))
        for chunks in (3, 16):
            got = flash_attn_func_host(qh, kh, vh, True, chunks=chunks, min_chunk_bytes=0)
            assert torch.equal(got, want), (b, s, h, hk, d, dtype, chunks)
    release_workspaces()
    assert torch.equal(flash_attn_func_host(qh, kh, vh, True, chunks=4, min_chunk_bytes=0), want)


def test_host_streaming_concurrent_callers():
    """Calls from several host threads on one device share its workspace
    one at a time and each gets its own results."""
    import threading

    from flash_attention import flash_attn_func, flash_attn_func_host

    cases = [make_inputs(4, 256, 2, 64, torch.float16, seed=90 + i) for i in range(4)]
    want = [flash_attn_func(q.cuda(), k.cuda(), v.cuda(), False).cpu() for q, k, v in cases]
    pinned = [tuple(t.pin_memory() for t in c) for c in cases]
    got, errors = [None] * 4, []

    def work(i):
        try:
            for _ in range(3):
                got[i] = flash_attn_func_host(*pinned[i], False, chunks=2, min_chunk_bytes=0)
        except Exception as e:  # noqa: BLE001 - reported by the main thread
            errors.append(e)

    threads = [threading.Thread(target=work, args=(i,)) for i in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    assert all(torch.equal(g, w) for g, w in zip(got, want))


def test_host_streaming_rejects_device_tensors():
    from flash_attention import flash_attn_func_host

    x = torch.zeros(1, 8, 2, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="must be a CPU tensor"):
        flash_attn_func_host(x, x, x)
