"""The model around the hot path (the reference's tests/test_verify_rollback.py and
tests/test_end_to_end.py structure, on a reduced random-init model): a multi-row verify step
equals the same rows as single steps, the rollback leaves every cache where single steps
would, the captured decode graphs give the eager loop's tokens exactly, and dense / sparse /
MTP greedy decoding agree."""
import pytest
import torch

from conftest import f32_np, rel_err

from hsd_b200.model import ModelArgs, MTPHead, NemotronModel, identical_prefix

B, N = 4, 2            # verify rows, rollback target (tests/test_verify_rollback.py:308-309)
BOUND = 5e-2           # the reference's bf16-level bounds for residuals and caches


def compare_states(model, sa, sb):
    assert int(sa.pos.item()) == int(sb.pos.item())
    o = int(sa.pos.item())
    diff = {"mamba_state": 0.0, "conv": 0.0, "kv": 0.0}
    mag = {"mamba_state": 1e-12, "conv": 1e-12, "kv": 1e-12}
    for l, t in enumerate(model.types):
        if t == "mamba":
            for a, b, k in zip(sa.mamba_now(l), sb.mamba_now(l), ("conv", "mamba_state")):
                diff[k] = max(diff[k], float((a.float() - b.float()).abs().max()))
                mag[k] = max(mag[k], float(b.float().abs().max()))
        elif t == "attention":
            for x, y in ((sa.kv[l].k[:, :o], sb.kv[l].k[:, :o]), (sa.kv[l].v[:, :o], sb.kv[l].v[:, :o])):
                diff["kv"] = max(diff["kv"], float((x.float() - y.float()).abs().max()))
                mag["kv"] = max(mag["kv"], float(y.float().abs().max()))
    worst = {k: diff[k] / mag[k] for k in diff}
    for k, v in worst.items():
        assert v < BOUND, (k, v)
    return worst


@pytest.fixture(scope="module")
def setup(cuda):
    model = NemotronModel(ModelArgs.tiny(), seed=3, device=cuda, mode="sparse", verify_rows=B)
    gen = torch.Generator(device=cuda).manual_seed(4)
    prompt = torch.randint(0, model.args.vocab, (20,), generator=gen, device=cuda)
    st0 = model.make_state()
    model.prefill(prompt, st0)
    cont = torch.randint(0, model.args.vocab, (B,), generator=gen, device=cuda)
    xin = model.embed(cont)
    return model, st0, xin


def single_steps(model, st0, xin, n):
    c = st0.clone()
    xs = [model.step(xin[i:i + 1], c) for i in range(n)]
    return torch.cat(xs), c


@pytest.mark.gpu
def test_verify_equals_b_single_steps(setup):
    model, st0, xin = setup
    xb, sb = single_steps(model, st0, xin, B)
    sa = st0.clone()
    xa = model.verify_step(xin, sa)
    model.rollback(sa, B, B)
    la, lb = model.logits(xa), model.logits(xb)
    assert torch.equal(la.argmax(-1), lb.argmax(-1))
    assert rel_err(f32_np(xa), f32_np(xb)) < BOUND
    compare_states(model, sa, sb)


@pytest.mark.gpu
def test_rollback_equals_n_single_steps(setup):
    model, st0, xin = setup
    _, sd = single_steps(model, st0, xin, N)
    se = st0.clone()
    model.verify_step(xin, se)
    model.rollback(se, N, B)
    compare_states(model, se, sd)


@pytest.mark.gpu
def test_rollback_then_single_steps(setup):
    model, st0, xin = setup
    _, sb = single_steps(model, st0, xin, B)
    sc = st0.clone()
    model.verify_step(xin, sc)
    model.rollback(sc, N, B)
    for i in range(N, B):
        model.step(xin[i:i + 1], sc)
    compare_states(model, sc, sb)


@pytest.mark.gpu
def test_graph_replay_equals_eager(cuda):
    """The captured step and the captured MTP iteration replay exactly the eager ops."""
    model = NemotronModel(ModelArgs.tiny(), seed=5, device=cuda, mode="sparse")
    gen = torch.Generator(device=cuda).manual_seed(6)
    prompt = torch.randint(0, model.args.vocab, (12,), generator=gen, device=cuda).tolist()
    eager, se = model.generate(prompt, 16, graphs=False)
    graph, sg = model.generate(prompt, 16, graphs=True)
    assert eager == graph
    assert se["margins"] == sg["margins"]
    mtp = MTPHead(model, seed=7)
    e2, _ = model.generate_mtp(prompt, mtp, n_draft=2, max_tokens=16, graphs=False)
    g2, _ = model.generate_mtp(prompt, mtp, n_draft=2, max_tokens=16, graphs=True)
    assert e2 == g2


@pytest.mark.gpu
def test_dense_sparse_mtp_greedy_tokens_identical(cuda):
    """Greedy tokens of sparse decoding, of MTP-2 speculative decoding and of dense decoding
    are identical -- exactly, not up to a near-tie: the sparse kernel reproduces the dense
    form bit for bit, and a verify row equals the token decoded alone (the reference's
    tests/test_end_to_end.py:56-97 allow divergence after 10 tokens)."""
    model = NemotronModel(ModelArgs.tiny(), seed=11, device=cuda, mode="dense")
    model.prefill_gemm = False
    gen = torch.Generator(device=cuda).manual_seed(12)
    prompt = torch.randint(0, model.args.vocab, (16,), generator=gen, device=cuda).tolist()
    dense, _ = model.generate(prompt, 32)
    model.set_mode("sparse")
    sparse, _ = model.generate(prompt, 32)
    assert dense == sparse
    mtp = MTPHead(model, seed=13)
    spec, st = model.generate_mtp(prompt, mtp, n_draft=2, max_tokens=32)
    assert spec == sparse
    assert st["steps"] >= 1 and sum(st["accepted_hist"]) == st["steps"]
    # forced acceptance: drafts replayed from the greedy run are all accepted
    rep, sr = model.generate_mtp(prompt, mtp, n_draft=2, max_tokens=32, replay=sparse)
    assert rep == sparse
    assert sr["accepted_hist"][2] == sr["steps"] - (1 if (32 - 1) % 3 else 0)
    model.set_mode("dense")
    spec_d, _ = model.generate_mtp(prompt, mtp, n_draft=2, max_tokens=32)
    assert spec_d == dense


@pytest.mark.gpu
def test_stock_and_gemm_prefill_agree_to_a_near_tie(cuda):
    """The checkpoint-layout dense kernel and the tensor-core prefill compute in other
    orders, so their tokens agree until an argmax near-tie (the reference's bound: 10)."""
    model = NemotronModel(ModelArgs.tiny(), seed=11, device=cuda, mode="stock")
    gen = torch.Generator(device=cuda).manual_seed(12)
    prompt = torch.randint(0, model.args.vocab, (16,), generator=gen, device=cuda).tolist()
    stock, st = model.generate(prompt, 24)
    model.set_mode("sparse")
    sparse, _ = model.generate(prompt, 24)
    n = identical_prefix(stock, sparse)
    assert n >= 10 or min(st["margins"][:n + 1]) < 0.05, (n, stock, sparse)
