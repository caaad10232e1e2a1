"""The model around the hot path (the reference's tests/test_verify_rollback.py and
tests/test_end_to_end.py structure, on a reduced random-init model): a multi-row verify step
equals the same rows as single steps, the rollback leaves every cache where single steps
would, and dense / sparse / MTP greedy decoding agree."""
import pytest
import torch

from conftest import f32_np, rel_err

from hsd_b200.model import KVCache, ModelArgs, MTPHead, NemotronModel

B, N = 4, 2            # verify rows, rollback target (tests/test_verify_rollback.py:308-309)
BOUND = 5e-2           # the reference's bf16-level bounds for residuals and caches


def clone_cache(cache):
    out = []
    for c in cache:
        if c is None:
            out.append(None)
        elif isinstance(c, KVCache):
            out.append(c.clone())
        else:
            out.append([None if t is None else t.clone() for t in c])
    return out


def compare_caches(model, ca, cb):
    diff = {"mamba_state": 0.0, "conv": 0.0, "kv": 0.0}
    mag = {"mamba_state": 1e-12, "conv": 1e-12, "kv": 1e-12}
    for l, t in enumerate(model.types):
        if t == "mamba":
            for i, k in ((0, "conv"), (1, "mamba_state")):
                a, b = ca[l][i].float(), cb[l][i].float()
                diff[k] = max(diff[k], float((a - b).abs().max()))
                mag[k] = max(mag[k], float(b.abs().max()))
        elif t == "attention":
            assert ca[l].offset == cb[l].offset
            o = ca[l].offset
            for x, y in ((ca[l].k[:o], cb[l].k[:o]), (ca[l].v[:o], cb[l].v[:o])):
                diff["kv"] = max(diff["kv"], float((x.float() - y.float()).abs().max()))
                mag["kv"] = max(mag["kv"], float(y.float().abs().max()))
    worst = {k: diff[k] / mag[k] for k in diff}
    for k, v in worst.items():
        assert v < BOUND, (k, v)
    return worst


@pytest.fixture(scope="module")
def setup(cuda):
    model = NemotronModel(ModelArgs.tiny(), seed=3, device=cuda, mode="sparse")
    gen = torch.Generator(device=cuda).manual_seed(4)
    prompt = torch.randint(0, model.args.vocab, (20,), generator=gen, device=cuda)
    cache0 = model.make_cache()
    model.prefill(prompt, cache0)
    cont = torch.randint(0, model.args.vocab, (B,), generator=gen, device=cuda)
    xin = model.embed(cont)
    return model, cache0, xin


def single_steps(model, cache0, xin, n):
    c = clone_cache(cache0)
    xs = [model.step(xin[i:i + 1], c) for i in range(n)]
    return torch.cat(xs), c


@pytest.mark.gpu
def test_verify_equals_b_single_steps(setup):
    model, cache0, xin = setup
    xb, cb = single_steps(model, cache0, xin, B)
    ca = clone_cache(cache0)
    xa = model.verify_step(xin, ca)
    la, lb = model.logits(xa), model.logits(xb)
    assert torch.equal(la.argmax(-1), lb.argmax(-1))
    assert rel_err(f32_np(xa), f32_np(xb)) < BOUND
    compare_caches(model, ca, cb)


@pytest.mark.gpu
def test_rollback_equals_n_single_steps(setup):
    model, cache0, xin = setup
    _, cd = single_steps(model, cache0, xin, N)
    ce = clone_cache(cache0)
    model.verify_step(xin, ce)
    model.rollback(ce, N, B)
    compare_caches(model, ce, cd)


@pytest.mark.gpu
def test_rollback_then_single_steps(setup):
    model, cache0, xin = setup
    _, cb = single_steps(model, cache0, xin, B)
    cc = clone_cache(cache0)
    model.verify_step(xin, cc)
    model.rollback(cc, N, B)
    for i in range(N, B):
        model.step(xin[i:i + 1], cc)
    compare_caches(model, cc, cb)


@pytest.mark.gpu
def test_dense_sparse_mtp_greedy_agree(cuda):
    """Dense and sparse down projections give the same greedy tokens, and MTP speculative
    decoding gives plain sparse decoding's tokens (tests/test_end_to_end.py:56-97: the
    reference allows divergence after 10 tokens on an argmax near-tie)."""
    model = NemotronModel(ModelArgs.tiny(), seed=11, device=cuda, mode="dense")
    gen = torch.Generator(device=cuda).manual_seed(12)
    prompt = torch.randint(0, model.args.vocab, (16,), generator=gen, device=cuda).tolist()
    dense, _ = model.generate(prompt, 24)
    model.set_mode("sparse")
    sparse, _ = model.generate(prompt, 24)
    same = next((i for i in range(24) if dense[i] != sparse[i]), 24)
    assert same >= 10, (same, dense, sparse)
    mtp = MTPHead(model, seed=13)
    spec, st = model.generate_mtp(prompt, mtp, n_draft=2, max_tokens=24)
    same2 = next((i for i in range(24) if spec[i] != sparse[i]), 24)
    assert same2 >= 10, (same2, spec, sparse)
    assert st["steps"] >= 1 and sum(st["accepted_hist"]) == st["steps"]
