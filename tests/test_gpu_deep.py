"""GPU checks of the multi-layer stack over one shared vals arena
(old/lib_sparse/prepare.py:50-148): the sparse stack against the dense
baseline within the bf16 tolerance 2e-2 (elementwise, absolute floor scaled
to the tensor's largest magnitude), the arena cursor chained across layers,
and the memory the sparse stack saves."""
import pytest
import torch

import autoresearch2_b200 as sf
from autoresearch2_b200 import deep

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _status():
    yield
    sf.check_status()


def inputs(tokens, hidm, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.randn(tokens, hidm, generator=g, device=DEV, dtype=torch.bfloat16)


def grads_of(model, x, sparse):
    model.zero_grad()
    sf.reset_sparse_globals()
    y = model.forward_sparse(x, sf.get_globals()) if sparse else model.forward_base(x)
    (y - x).float().pow(2).mean().backward()
    return [y.detach()] + [p.grad.clone() for p in model.parameters()]


def assert_close(got, want, tol=2e-2):
    for g, w in zip(got, want):
        err = (g.float() - w.float()).abs().max().item()
        assert err <= tol * w.float().abs().max().item(), err


@pytest.mark.parametrize("act", ["relu", "relu2"])
def test_sparse_stack_matches_dense(act):
    T, H, L = 1024, 256, 3
    model = deep.DeepFFN(torch.bfloat16, layers=L, hidm=H, act=act)
    x = inputs(T, H)
    sf.init_sparse_buffer(deep.arena_elements(T, H, L, fill=1.0), DEV, torch.bfloat16)
    got = grads_of(model, x, sparse=True)
    if act == "relu":
        want = grads_of(model, x, sparse=False)
    else:  # the dense baseline is ReLU; ReLU^2 against torch autograd of the same stack
        model.zero_grad()
        h = x
        for W1, W2 in zip(model.W1s, model.W2s):
            z = torch.relu(torch.nn.functional.rms_norm(h, h.shape[-1:]) @ W1.T)
            h = h + (z * z) @ W2.T
        (h - x).float().pow(2).mean().backward()
        want = [h.detach()] + [p.grad.clone() for p in model.parameters()]
    assert_close(got, want)


def test_arena_cursor_chains_across_layers():
    """Each layer appends its activation's nonzeros behind the previous
    layer's; run_step rewinds the cursor, so two steps give the same loss."""
    T, H, L = 512, 256, 4
    model = deep.DeepFFN(torch.bfloat16, layers=L, hidm=H)
    x = inputs(T, H, seed=1)
    buf = sf.init_sparse_buffer(deep.arena_elements(T, H, L), DEV, torch.bfloat16)
    h = x
    for W1, W2 in zip(model.W1s, model.W2s):
        before = buf.used()
        out = sf.FFNSparse.apply(torch.nn.functional.rms_norm(h, h.shape[-1:]), W1, W2,
                                 buf.as_sparse_data())
        z = out.grad_fn.z_sparse
        assert int(z.vals_offset.item()) == before
        assert buf.used() - before == int(z.prefix[-1].item()) > 0
        h = h + out
    loss1 = deep.run_step(x, model, sparse=True)[0]
    loss2 = deep.run_step(x, model, sparse=True)[0]
    assert torch.equal(loss1, loss2)


def test_memory_report_shows_the_saving():
    """Eight layers, 8192 tokens, width 512: the dense baseline keeps eight
    dense ReLU outputs, the sparse stack one arena of 0.55 of that plus masks."""
    model = deep.DeepFFN(torch.bfloat16, layers=8, hidm=512)
    r = deep.memory_report(inputs(8192, 512, seed=2), model)
    assert r["sparse"]["peak_mb"] < r["dense"]["peak_mb"], r
    assert 0 < r["arena"]["used_fraction"] <= 1
    assert 0.4 < r["arena"]["activation_zeros"] < 0.6
    assert r["loss_rel_diff"] < 2e-2 and r["grad_std_rel_diff"] < 5e-2, r
    # no arena: each layer's values exactly sized and freed after its backward
    e = r["sparse_exact"]
    assert e["peak_mb"] < r["sparse"]["peak_mb"], r
    assert e["loss_rel_diff"] == r["loss_rel_diff"] and e["grad_std_rel_diff"] == r["grad_std_rel_diff"], r


def test_exact_size_values_without_an_arena():
    """FFNSparse / FFNSpRelu2 given no arena keep each layer's z in a values
    tensor of exactly its nnz: the same output, gradients and packed z as the
    same layer over an arena (bit for bit), vals sized to prefix[-1]."""
    import autoresearch2_b200 as sf
    for fn in (sf.FFNSparse, sf.FFNSpRelu2):
        x = inputs(1000, 512, seed=5).requires_grad_()
        model = deep.DeepFFN(torch.bfloat16, layers=1, hidm=512)
        W1, W2 = model.W1s[0], model.W2s[0]
        arena = (torch.empty(1000 * W1.shape[0], dtype=torch.bfloat16, device="cuda"),
                 torch.zeros(1, dtype=torch.int32, device="cuda"))
        outs, grads = [], []
        for sd in (arena, None):
            y = fn.apply(x, W1, W2, sd)
            z = y.grad_fn.z_sparse
            if sd is None:
                assert z.vals.numel() == int(z.prefix[-1].item()) > 0
                assert z.vals.untyped_storage().nbytes() == z.vals.numel() * 2
            else:
                packed = z.vals[:int(z.prefix[-1].item())].clone()
            outs.append((y.detach().clone(), z.vals[:int(z.prefix[-1].item())].clone()))
            g = torch.randn_like(y)
            grads.append(torch.autograd.grad(y, (x, W1, W2), g if not grads else grads[0][3]))
            grads[-1] = (*grads[-1], g)
        assert torch.equal(outs[0][0], outs[1][0])
        assert torch.equal(outs[1][1].view(torch.int16), packed.view(torch.int16))
        for a, b in zip(grads[0][:3], grads[1][:3]):
            assert torch.equal(a, b)
    sf.check_status()
