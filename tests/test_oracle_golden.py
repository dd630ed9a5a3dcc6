"""CPU: the numpy oracle against golden outputs of the reference's own code.

The fixtures in tests/golden/ were produced by running the reference's
functions on CPU (tests/golden/make_golden.py). These tests pin the oracle
that the GPU parity tests then use as their checker.
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import muon as om
from oracle.bf16 import from_bits, rel_fro, round_bf16, to_bits

GOLD = Path(__file__).parent / "golden"


@pytest.fixture(scope="module")
def mz():
    return np.load(GOLD / "muon_golden.npz")


def test_round_bf16_known_values():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5, 3.4445, 0.0, -0.0, np.inf, np.nan], dtype=np.float32)
    r = round_bf16(x)
    assert r[0] == 1.0 and r[1] == 1.0  # tie to even
    assert r[2] == np.float32(1.0078125)
    assert r[3] == -2.5 and r[4] == np.float32(3.4375)
    assert np.isinf(r[7]) and np.isnan(r[8])
    assert np.array_equal(from_bits(to_bits(r[:8])), r[:8])
    assert round_bf16(np.float32(1.0)).shape == ()


def test_ns_serial_small_shapes(mz):
    for i, (r, c) in enumerate(mz["serial_shapes"]):
        G = from_bits(mz[f"serial{i}_in"]).reshape(r, c)
        ref = from_bits(mz[f"serial{i}_out"]).reshape(r, c)
        assert rel_fro(om.zeropower(G, 5, 1e-7), ref) < 2e-2, (r, c)


def test_ns_batched(mz):
    X = from_bits(mz["batched_in"]).reshape(3, 64, 192)
    ref = from_bits(mz["batched_out"]).reshape(3, 64, 192)
    assert rel_fro(om.zeropower(X, 5, 1e-7, orient=False), ref) < 2e-2


@pytest.mark.parametrize("steps", [0, 1, 3])
def test_ns_step_counts(mz, steps):
    G = from_bits(mz["steps_in"]).reshape(48, 160)
    ref = from_bits(mz[f"steps{steps}_out"]).reshape(48, 160)
    err = rel_fro(om.zeropower(G, steps, 1e-7), ref)
    assert err < (1e-6 if steps == 0 else 2e-2)


def test_ns_config1_shape(mz):
    torch = pytest.importorskip("torch")
    g0 = torch.Generator().manual_seed(0)
    for name, (r, c) in (("cfg1_wide", (768, 3072)), ("cfg1_tall", (3072, 768))):
        G = (torch.randn(r, c, generator=g0) * 0.02).to(torch.bfloat16).float().numpy()
        sums = [G.astype(np.float64).sum(), (G.astype(np.float64) ** 2).sum()]
        assert np.allclose(sums, mz[f"{name}_in_sums"]), "torch CPU RNG changed"
        O = om.zeropower(G, 5, 1e-7)
        assert rel_fro(O[:64], from_bits(mz[f"{name}_out_rows"]).reshape(64, -1)) < 2e-2
        assert rel_fro(O.astype(np.float64).sum(0), mz[f"{name}_out_colsum"]) < 2e-2
        assert abs(np.linalg.norm(O) - mz[f"{name}_out_fro"][0]) / mz[f"{name}_out_fro"][0] < 1e-3


def test_adjusted_lr(mz):
    for (lr, r, c), o, m, n in zip(mz["lr_cases"], mz["lr_original"], mz["lr_match"], mz["lr_none"]):
        assert om.adjusted_muon_lr(lr, (int(r), int(c)), "original") == pytest.approx(o)
        assert om.adjusted_muon_lr(lr, (int(r), int(c)), "match_rms_adamw") == pytest.approx(m)
        assert om.adjusted_muon_lr(lr, (int(r), int(c)), "none") == pytest.approx(n)
    with pytest.raises(ValueError):
        om.adjusted_muon_lr(0.02, (2, 3), "bogus")


NAMES = [("h.0.attn.c_attn.weight", (64, 192)), ("h.0.attn.c_proj.weight", (64, 64)),
         ("h.0.mlp.c_fc.weight", (64, 256)), ("h.0.mlp.c_proj.weight", (256, 64)),
         ("h.1.mlp.c_fc.weight", (64, 256)), ("h.1.mlp.c_proj.weight", (256, 64))]


@pytest.mark.parametrize("mode", ["batched", "serial"])
def test_muon_two_steps(mz, mode):
    P = [from_bits(mz[f"muon_init_{n}"]).reshape(s) for n, s in NAMES]
    M = [np.zeros(s, np.float32) for _, s in NAMES]
    P0 = [p.copy() for p in P]
    for step in range(2):
        G = [from_bits(mz[f"muon_grad{step}_{n}"]).reshape(s) for n, s in NAMES]
        P, M = om.muon_step(P, G, M, lr=0.02, mu=0.95, nesterov=True, wd=0.01, ns_steps=5, eps=1e-7)
    for (n, s), p, m, p0 in zip(NAMES, P, M, P0):
        ref = from_bits(mz[f"muon_{mode}_{n}"]).reshape(s)
        assert rel_fro(p - p0, ref - p0) < 0.1, n
        assert np.array_equal(m, from_bits(mz[f"muon_{mode}_mom_{n}"]).reshape(s)), n


def test_ns_flops_config4():
    shapes = [(1600, 4800), (1600, 1600), (1600, 6400), (6400, 1600)] * 48
    total = sum(om.ns_flops(min(s), max(s)) for s in shapes)
    assert abs(total / 1e12 - 55.05) < 0.01


# ---------------------------------------------------------------- Kronecker oracle
def test_kron_oracle_matches_reference_golden():
    from oracle import kron as ok
    z = np.load(GOLD / "kron_golden.npz")
    for i in range(3):
        Y = ok.kron_apply_shared_2d(z[f"apply{i}_X"], z[f"apply{i}_A"], z[f"apply{i}_B"])
        assert rel_fro(Y, z[f"apply{i}_Y"]) < 1e-6
    for i in range(2):
        Y = ok.kron_sum(z[f"ksum{i}_X"], z[f"ksum{i}_A"], z[f"ksum{i}_B"])
        assert rel_fro(Y, z[f"ksum{i}_Y"]) < 1e-6
    for S in (1, 2, 4):
        X, A, B = z[f"multi{S}_X"], z[f"multi{S}_A"], z[f"multi{S}_B"]
        Y = ok.kron_apply(X, A, B)
        assert rel_fro(Y, z[f"multi{S}_Y"]) < 1e-6
        W = ok.dense_operator(A, B)
        Yd = (X.reshape(X.shape[0], -1).astype(np.float64) @ W.T).reshape(X.shape)
        assert rel_fro(Yd, z[f"multi{S}_Ydense"]) < 1e-6


# ---------------------------------------------------------------- Shampoo oracle
def test_coupled_newton_matches_reference_golden():
    from oracle import shampoo as osh
    z = np.load(GOLD / "newton_golden.npz")
    for i in range(2):
        A = z[f"newton{i}_A"]
        for root in (2, 4):
            X, it, err = osh.coupled_newton_one(A, root)
            assert rel_fro(X, z[f"newton{i}_root{root}"]) < 1e-4
            # and it is the inverse root
            assert rel_fro(np.linalg.matrix_power(X, root) @ A, np.eye(A.shape[0])) < 1e-4
            assert rel_fro(X, osh.inverse_root(A, root)) < 1e-4


def test_gpt2xl_soap_blocks():
    """GPT-2-XL blocked at max_preconditioner_dim 1024: 42 blocks per layer in 10 block shapes,
    2016 blocks over the 48 layers."""
    import collections
    from oracle import shampoo as osh
    assert osh.block_sizes(1600, 1024) == [1024, 576]
    assert osh.block_sizes(4800, 1024) == [1024] * 4 + [704]
    assert osh.block_sizes(6400, 1024) == [1024] * 6 + [256]
    cnt = collections.Counter()
    for r, c in [(1600, 4800), (1600, 1600), (1600, 6400), (6400, 1600)]:
        for rb in osh.block_sizes(r, 1024):
            for cb in osh.block_sizes(c, 1024):
                cnt[(rb, cb)] += 1
    assert sum(cnt.values()) == 42
    assert cnt[(1024, 1024)] == 17 and cnt[(576, 1024)] == 11 and cnt[(1024, 576)] == 7
    total = 48 * sum(osh.soap_flops(r, c) * k for (r, c), k in cnt.items())
    assert abs(total / 1e12 - 16.29) < 0.01


def test_reconstruct_oracle_matches_reference_golden():
    from oracle import kron as ok
    z = np.load(GOLD / "kronrec_golden.npz")
    for S in (1, 7, 64):
        for K in (5, 4, 3):
            fs = [z[f"S{S}_K{K}_f{i}"] for i in range(K)]
            W = ok.reconstruct(fs)
            assert W.shape == (16, 768)
            assert rel_fro(W, z[f"S{S}_K{K}_W"]) < 1e-5


def test_coupled_newton_batched_golden():
    """The oracle's per-factor recurrence against the reference's batched_coupled_newton
    (per-factor mask) on SPD batches with a hard (small-ridge) tail."""
    from oracle import shampoo as osh
    z = np.load(GOLD / "newton_golden.npz")
    for j, roots in ((0, (2, 4)), (1, (4,))):
        A = z[f"nbatch{j}_A"]
        for root in roots:
            for b in range(A.shape[0]):
                X, it, err = osh.coupled_newton_one(A[b], root)
                ref_it = int(z[f"nbatch{j}_root{root}_iters"][b])
                assert abs(it - ref_it) <= 1, (j, root, b, it, ref_it)
                assert int(z[f"nbatch{j}_root{root}_iters_one"][b]) == ref_it
                hard = b == A.shape[0] - 1
                assert rel_fro(X, z[f"nbatch{j}_root{root}_X"][b]) < (2e-2 if hard else 1e-4), (j, root, b)
