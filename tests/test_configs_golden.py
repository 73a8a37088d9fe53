"""The oracle against the reference's 8B-shape fixtures (CPU).

make_weights' streaming form (on_layer) draws the same weights as the
all-at-once form; and the oracle at TP8 reproduces the reference's TP8 layer
(config 3: one 8B-shape layer, batch 4) on the 512-token prefill and the
first decode steps, within the tolerance of the two bf16 all-reduce orders."""
import torch

from oracle import decoder as odec
from tests.golden import cases
from tests.helpers import as_tensor, compare, load_golden


def test_streamed_weights_match_make_weights():
    spec = odec.Spec(hidden=256, q_heads=2, kv_heads=1, inter=512, vocab=64, layers=3)
    whole = odec.make_weights(spec, seed=4, random_norms=True)
    kept = []
    streamed = odec.make_weights(spec, seed=4, random_norms=True,
                                 on_layer=lambda i, lw: kept.append(i) or {"i": i, **lw})
    assert kept == [0, 1, 2]
    for a, b in zip(whole["layers"], streamed["layers"]):
        for k, v in a.items():
            assert torch.equal(v, b[k]), k
    for k in ("embed", "final_norm", "lm_head"):
        assert torch.equal(whole[k], streamed[k])


def test_oracle_layer_tp8_matches_reference_fixture():
    cfg = cases.LAYER_TP8
    g = load_golden("layer8b_tp8")
    c = cases.layer_tp8_case()
    assert cases.weights_checksum(c["weights"]) == float(g["weights_checksum"])
    o = odec.OracleDecoder(c["spec"], c["weights"], tp=cfg["tp"])
    kv = o.init_kv_cache(cfg["B"])
    R = cases.fingerprint_matrix(cfg["proj_dim"])
    with torch.no_grad():
        pre = o.forward_layer(c["hidden"], 0, kv, 0)
        n = 4   # the first decode steps (the GPU test runs all 128)
        steps = torch.stack([o.forward_layer(c["dec_in"][i], 0, kv, cfg["S"] + i)
                             for i in range(n)])
    compare("oracle prefill fingerprint", cases.layer_fingerprint(pre, c["hidden"], R),
            as_tensor(g["pre_fp"]), max_abs=2e-2, rel_scale=True, min_cos=0.9999)
    compare("oracle prefill rows", pre[:, list(cfg["pre_tokens"])], as_tensor(g["pre_rows"]),
            max_abs=3e-2, rel_scale=True, min_cos=0.9999)
    compare("oracle decode fingerprint", cases.layer_fingerprint(steps, c["dec_in"][:n], R),
            as_tensor(g["dec_fp"])[:n], max_abs=2e-2, rel_scale=True, min_cos=0.9999)
    compare("oracle decode row", steps[0], as_tensor(g["dec_rows"])[0], max_abs=3e-2,
            rel_scale=True, min_cos=0.9999)
