"""CPU: generated device headers are current, and the generated formulas match the oracle."""

import numpy as np

from flashns_b200 import codegen


def test_generated_headers_are_current():
    for path, text in codegen.outputs().items():
        assert path.read_text() == text, f"{path.name} is stale: run python -m flashns_b200.codegen"


def test_uvp_polynomials_match_reference_residual_table():
    """The nine generated (u, v, p) residuals equal ns_seed.residual_terms
    (src/flashns/ns_seed.py:26-43) term by term, evaluated on random jets."""
    g = np.load(__import__("tests.cases", fromlist=["GOLDEN"]).GOLDEN / "reference_seed.npz")
    from oracle import residuals as RS
    for k in range(int(g["seed_count"])):
        p = f"seed{k}_"
        nu, gamma = (float(v) for v in g[p + "nu_gamma"])
        jets = g[p + "jets"]
        res, _ = codegen.residuals_uvp()
        lookup = {a: i for i, a in enumerate(codegen.basis(2))}
        from math import factorial, prod
        values = np.zeros((len(jets), len(res)))
        y = jets.reshape(len(jets), 30)
        for r, expr in enumerate(res):
            for key, (a, b) in expr.items():
                term = np.full(len(jets), a + b * nu)
                for f, al in key:
                    term = term * prod(factorial(v) for v in al) * y[:, lookup[al] * 3 + f]
                values[:, r] += term
        np.testing.assert_allclose(values, g[p + "res"], rtol=1e-11, atol=1e-12)
        np.testing.assert_allclose(values, RS.residual_values(jets, "uvp", nu, gamma), rtol=1e-11, atol=1e-12)


def test_head_output_lists_match_the_generated_seeds():
    """The register form of the two-group head forms only the output values the
    stream-function seed reads (HeadOutputs in eval.cu); that list must be exactly the
    y[...] inputs (and dy[...] outputs) of the generated seed formula, or the seed would
    read a value never formed."""
    import re
    from pathlib import Path
    csrc = Path(codegen.__file__).resolve().parent / "csrc"
    seeds = (csrc / "residual_generated.cuh").read_text()
    source = (csrc / "eval.cu").read_text()
    block = source[source.index("struct HeadOutputs"):source.index("hpp_smem_bytes")]
    lists = [[int(v) for v in m.split(",")] for m in re.findall(r"constexpr int v\[\w+\] = \{([^}]*)\}", block)]
    assert len(lists) == 1
    for name, listed in (("seed_psi_2d", lists[0]),):
        body = seeds[seeds.index(name + "("):]
        body = body[:body.index("\n}\n")]
        used = sorted({int(i) for i in re.findall(r"\by\[(\d+)\]", body)})
        seeded = sorted({int(i) for i in re.findall(r"\bdy\[(\d+)\] \+=", body)})
        assert listed == used == seeded, name
