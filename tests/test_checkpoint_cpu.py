"""SafeTensors ingestion on CPU: a synthetic MLX checkpoint written with the
reference's tensor names (sharded, with an index and per-module quantisation
overrides) loads back into the block's weight dict unchanged, drives the oracle
to the same outputs, and malformed shards fail with the reference's header
errors (expert_paging/safetensors_header.rs)."""
import json
import os
import struct

import numpy as np
import pytest

from astronomical_b200 import checkpoint as ck
from astronomical_b200 import synthetic
from oracle import oracle as O


def small_cfg():
    return dict(hidden=256, experts=8, top_k=2, intermediate=128, shared_intermediate=128,
                group=64, bits=4, normalize=True, zipf=None)


def write_checkpoint(tmp_path, layers, cfg, extra_quant=None, shards=2):
    names = {}
    for li, w in enumerate(layers):
        names.update(ck.export_moe_layer(w, li))
    keys = sorted(names)
    weight_map = {}
    for s in range(shards):
        part = {k: names[k] for k in keys[s::shards]}
        fn = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        ck.write_safetensors(os.path.join(tmp_path, fn), part, {"format": "mlx"})
        weight_map.update({k: fn for k in part})
    with open(os.path.join(tmp_path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": weight_map}, f)
    quant = {"group_size": cfg["group"], "bits": cfg["bits"], "mode": "affine"}
    for li, w in enumerate(layers):
        quant.update(ck.module_overrides(w, li))
    quant.update(extra_quant or {})
    config = {"model_type": "qwen3_5_moe", "quantization": quant, "quantization_config": quant,
              "text_config": {"hidden_size": cfg["hidden"], "num_experts": cfg["experts"],
                              "num_experts_per_tok": cfg["top_k"],
                              "moe_intermediate_size": cfg["intermediate"],
                              "shared_expert_intermediate_size": cfg["shared_intermediate"],
                              "norm_topk_prob": True}}
    with open(os.path.join(tmp_path, "config.json"), "w") as f:
        json.dump(config, f)
    return str(tmp_path)


@pytest.mark.parametrize("quant", [None, {"router": (8, 64), "shared_gate": (8, 64),
                                          "down": (8, 64), "sdown": (4, 32)}])
def test_checkpoint_round_trip_and_oracle(tmp_path, quant):
    cfg = small_cfg()
    layers = [synthetic.make_block_weights(cfg, seed=s, quant=quant) for s in (1, 2)]
    d = write_checkpoint(tmp_path, layers, cfg)
    c = ck.Checkpoint(d)
    assert c.block_config() == cfg
    x = synthetic.make_hidden_states(24, cfg["hidden"], seed=5)
    for li, w in enumerate(layers):
        got = c.moe_layer(li)
        want = {k: v for k, v in w.items() if k != "config"}
        assert set(k for k in got if k != "config") == set(want)
        for k, v in want.items():
            if isinstance(v, int):
                assert got[k] == v, k
            else:
                assert np.array_equal(np.asarray(got[k]), v), k
        y0, ids0, _ = O.moe_block_forward(w, x)
        y1, ids1, _ = O.moe_block_forward(got, x)
        assert np.array_equal(y0, y1) and np.array_equal(ids0, ids1)


def test_single_file_checkpoint_and_missing_tensor(tmp_path):
    cfg = small_cfg()
    w = synthetic.make_block_weights(cfg, seed=3)
    names = ck.export_moe_layer(w, 0)
    missing = "language_model.model.layers.0.mlp.switch_mlp.down_proj.scales"
    del names[missing]
    c = _single_file(tmp_path, names)
    with pytest.raises(ck.CheckpointError, match="down_proj"):
        c.moe_layer(0)


def _single_file(tmp_path, names, quant=None):
    ck.write_safetensors(os.path.join(tmp_path, "model.safetensors"), names)
    q = quant or {"group_size": 64, "bits": 4}
    with open(os.path.join(tmp_path, "config.json"), "w") as f:
        json.dump({"quantization": q,
                   "text_config": {"hidden_size": 256, "num_experts": 8, "num_experts_per_tok": 2,
                                   "moe_intermediate_size": 128,
                                   "shared_expert_intermediate_size": 128}}, f)
    return ck.Checkpoint(str(tmp_path))


def test_wrong_dtype_shape_and_quantisation_are_rejected(tmp_path):
    w = synthetic.make_block_weights(small_cfg(), seed=4)
    k = "language_model.model.layers.0.mlp.switch_mlp.gate_proj.weight"
    names = ck.export_moe_layer(w, 0)
    names[k] = ("I32", names[k][1].view(np.int32))
    with pytest.raises(ck.CheckpointError, match="dtype"):
        _single_file(tmp_path, names).moe_layer(0)
    names = ck.export_moe_layer(w, 0)
    names[k] = ("U32", names[k][1][:, :64])
    with pytest.raises(ck.CheckpointError, match="shape"):
        _single_file(tmp_path, names).moe_layer(0)
    # a config whose profile does not match the stored codes
    names = ck.export_moe_layer(w, 0)
    with pytest.raises(ck.CheckpointError, match="shape"):
        _single_file(tmp_path, names, {"group_size": 64, "bits": 8}).moe_layer(0)
    with pytest.raises(ck.CheckpointError, match="unsupported quantisation"):
        _single_file(tmp_path, names, {"group_size": 48, "bits": 4}).moe_layer(0)
    # quantisation copies that disagree
    cfgj = json.load(open(os.path.join(tmp_path, "config.json")))
    cfgj["quantization_config"] = dict(cfgj["quantization"], bits=8)
    json.dump(cfgj, open(os.path.join(tmp_path, "config.json"), "w"))
    with pytest.raises(ck.CheckpointError, match="differ"):
        ck.Checkpoint(str(tmp_path))


def _raw_shard(path, header_bytes, payload=b""):
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(header_bytes)))
        f.write(header_bytes)
        f.write(payload)


def test_header_validation(tmp_path):
    p = os.path.join(tmp_path, "x.safetensors")
    with open(p, "wb") as f:
        f.write(b"\x01\x02")
    with pytest.raises(ck.SafetensorsHeaderError, match="too small"):
        ck.read_header(p)
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", ck.MAXIMUM_HEADER_BYTES + 1))
    with pytest.raises(ck.SafetensorsHeaderError, match="safety limit"):
        ck.read_header(p)
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", 100) + b"{}")
    with pytest.raises(ck.SafetensorsHeaderError, match="beyond the file"):
        ck.read_header(p)
    _raw_shard(p, b"[1, 2]")
    with pytest.raises(ck.SafetensorsHeaderError, match="JSON object"):
        ck.read_header(p)
    _raw_shard(p, b"{not json")
    with pytest.raises(ck.SafetensorsHeaderError, match="valid JSON"):
        ck.read_header(p)
    _raw_shard(p, json.dumps({"t": {"dtype": "Q7", "shape": [1], "data_offsets": [0, 1]}}).encode(),
               b"\0")
    with pytest.raises(ck.SafetensorsHeaderError, match="unsupported dtype"):
        ck.read_header(p)
    _raw_shard(p, json.dumps({"t": {"dtype": "U32", "shape": [2], "data_offsets": [0, 4]}}).encode(),
               b"\0" * 4)
    with pytest.raises(ck.SafetensorsHeaderError, match="need 8"):
        ck.read_header(p)
    _raw_shard(p, json.dumps({"t": {"dtype": "U32", "shape": [2], "data_offsets": [0, 8]}}).encode(),
               b"\0" * 4)
    with pytest.raises(ck.SafetensorsHeaderError, match="beyond"):
        ck.read_header(p)
    with pytest.raises(ck.SafetensorsHeaderError, match="does not exist"):
        ck.read_header(os.path.join(tmp_path, "absent.safetensors"))
    # a valid one reads back, metadata skipped
    _raw_shard(p, json.dumps({"__metadata__": {"format": "mlx"},
                              "t": {"dtype": "U32", "shape": [2], "data_offsets": [0, 8]}}).encode(),
               struct.pack("<II", 7, 9))
    h = ck.read_header(p)
    assert list(h) == ["t"] and ck.open_tensor(p, h["t"]).tolist() == [7, 9]
