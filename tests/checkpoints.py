"""Seeded synthetic float checkpoints (.npz, the layout the reference's training saves, yggdrasil/model.py:154-158) and
export records (the `stats` / `quantize` fields of cpu/export.py:563-572) for the .npz -> int8 tests. The datasets
and released checkpoints are absent here; random parameters of the right shapes stand in."""
import json

import numpy as np

OLD = {"token_layer": "root", "routed_layers": "branches", "output_bias": "head_b", "token_embed": "v_tok",
       "input_proj": "u_in", "bias": "c", "readout": "p_out", "unembed": "q_out", "rotation": "skew",
       "decay": "d_raw", "router_embed": "tok", "router_weight": "w_node", "router_bias": "b_node",
       "layer_input_down": "v_low", "layer_input_proj": "u_low"}

SHAPE = dict(vocab=27, n=64, block=16, depth=4, readout=8, layer_input=16, input_rank=16, router_token=8, routed=2)


def synthetic_checkpoint(path, seed=0, old_keys=False, shape=SHAPE):
    """Write a random checkpoint: a token layer and `routed` routed layers."""
    rng = np.random.default_rng(seed)
    V, n, b, D, R, R2, k, F = (shape[x] for x in ("vocab", "n", "block", "depth", "readout", "layer_input",
                                                   "input_rank", "router_token"))
    flat = {}

    def layer(prefix, E, routed):
        p = {"token_embed": rng.normal(0, 1, (V, k)), "input_proj": rng.normal(0, 0.3, (E, n, k)),
             "bias": rng.normal(0, 0.5, (E, n)), "rotation": rng.normal(0, 0.4, (E, n // b, b, b)),
             "decay": rng.uniform(0.6, 1.05, (E, n)), "readout": rng.normal(0, shape.get("readout_std", 0.2), (E, R, n)),
             "unembed": rng.normal(0, shape.get("unembed_std", 0.3), (V, R))}
        if routed:
            p.update(router_embed=rng.normal(0, 1, (V, F)), router_weight=rng.normal(0, 0.3, (E - 1, F + n)),
                     router_bias=rng.normal(0, 0.1, E - 1), layer_input_down=rng.normal(0, 0.2, (R2, n)),
                     layer_input_proj=rng.normal(0, 0.2, (E, n, R2)))
        for key, v in p.items():
            flat[f"{prefix}/{key}"] = v.astype(np.float32)

    layer("token_layer", V, False)
    for i in range(shape["routed"]):
        layer(f"routed_layers/{i}", 2 ** D, True)
    flat["output_bias"] = rng.normal(0, 0.5, V).astype(np.float32)
    if old_keys:
        flat = {"/".join(OLD.get(p, p) for p in name.split("/")): v for name, v in flat.items()}
    np.savez(path, **flat)


def synthetic_record(seed=0, hmargin=0.85, group=False, factored=False, shape=SHAPE):
    """An export record with positive calibration maxima for every layer."""
    rng = np.random.default_rng(1000 + seed)
    n, R = shape["n"], shape["readout"]
    stats = []
    for _ in range(1 + shape["routed"]):
        g = rng.uniform(1.0, 6.0, n // 16)
        stats.append(dict(state_max=float(g.max()), layer_input_max=float(rng.uniform(2, 5)),
                          readout_max=float(rng.uniform(4, 9)), state_group_max=g.tolist(),
                          readout_row_max=rng.uniform(2, 9, R).tolist()))
    return dict(quantize=dict(hmargin=hmargin, group=group, factored=factored), stats=stats,
                storage="factored" if factored else "table", state_scale="group" if group else "tensor")


def write_record(path, **kw):
    with open(path, "w") as f:
        json.dump(synthetic_record(**kw), f)
