"""A decode model read from a model directory in the reference's layout (CPU only): the
tiny dense, MoE and MLA configurations written with the reference's writers restated
(tensor names of crates/soso-llm-core/src/layer.rs, manifest of manifest.rs) come back as
the same DenseConfig and the same tensor bytes."""
import dataclasses

import numpy as np
import pytest

import oracle
from soso_b200 import decode
from soso_b200.formats import DTYPE_F32
from soso_b200.som import SomError
from soso_b200.som_load import load_decode_model

KIND_IDX = {"gqa": 0, "mla": 1, "dense": 0, "moe": 1}


def som_name(key: str) -> str:
    if key == "token_embd":
        return "embed"
    if key == "output":
        return "lm_head"
    if not key.startswith("blk."):
        return key
    _, l, rest = key.split(".", 2)
    if rest[0] == "E" and rest[1:4].isdigit():
        rest = f"E{int(rest[1:4]):02d}" + rest[4:]
    return f"L{int(l):02d}.{rest}"


def write_model(tmp, cfg, model, n_shared=0, version=5, v_dim=None, ext=None):
    (tmp / "shards").mkdir()
    entries = []
    H = cfg.hidden

    def put(name, data: bytes, dtype, shape):
        shard = name + ".tensor"
        (tmp / "shards" / shard).write_bytes(oracle.pack_shard(data))
        entries.append((len(entries), name, shard, 0, len(data), shape, dtype, 0))

    for key, arr in model.items():
        if key.endswith("qkv_bias"):
            l = int(key.split(".")[1])
            parts = np.split(arr, [cfg.q_dim, cfg.q_dim + cfg.kv_dim])
            for n, p in zip(("attn_q", "attn_k", "attn_v"), parts):
                put(f"L{l:02d}.{n}.bias", p.astype(np.float32).tobytes(), DTYPE_F32, (p.size,))
            continue
        kind = key.split(".")[-1]
        if arr.dtype == np.float32:
            put(som_name(key), arr.tobytes(), DTYPE_F32, (arr.size,))
            continue
        width = cfg.shared_ffn if ".S00." in key else cfg.moe_ffn
        shape = {"ffn_gate": (width, H), "ffn_up": (width, H), "ffn_down": (H, width)}.get(kind, (0, 0)) \
            if (".E" in key or ".S00." in key) else (1, 1)
        dt = cfg.dtypes["ffn_gate_inp" if kind == "ffn_gate_inp" else kind if kind in cfg.dtypes else
                        {"token_embd": "token_embd", "output": "output"}[kind]]
        put(som_name(key), arr.tobytes(), dt, shape)
    flags = (8 if cfg.neox else 0) | (16 if cfg.qk_norm else 0)
    specs = []
    for l in range(cfg.n_layers):
        moe = cfg.is_moe(l)
        specs.append((KIND_IDX["mla" if cfg.mla else "gqa"], KIND_IDX["moe" if moe else "dense"], cfg.heads,
                      cfg.kv_heads, cfg.ffn, cfg.kv_rank, cfg.q_rank, cfg.qk_rope, cfg.qk_nope,
                      cfg.v_dim if v_dim is None else v_dim,
                      cfg.n_exp if moe else 0, cfg.top_k if moe else 0, cfg.moe_ffn if moe else 0,
                      n_shared if moe else 0, flags))
    core = ("t", cfg.vocab, H, cfg.n_layers, cfg.heads, cfg.ffn, cfg.ctx, cfg.kv_heads, cfg.theta, cfg.eps,
            cfg.n_exp, cfg.top_k, cfg.moe_ffn)
    (tmp / "manifest.som").write_bytes(oracle.serialize_manifest(version, core, specs, [], ext=ext) if version > 5
                                       else oracle.serialize_manifest_prefix(version, core, specs, []))
    (tmp / "index.som").write_bytes(oracle.serialize_index(entries))


FIELDS = ("n_layers", "hidden", "heads", "kv_heads", "head_dim", "ffn", "vocab", "ctx", "theta", "neox", "qkv_bias",
          "qk_norm", "mla", "q_rank", "kv_rank", "qk_nope", "qk_rope", "v_dim", "n_exp", "top_k", "moe_ffn",
          "first_moe", "shared_ffn", "shared_gate")


@pytest.mark.parametrize("which", ["TINY", "TINY_MOE", "TINY_MLA"])
def test_round_trip(tmp_path, which):
    cfg = getattr(decode, which)
    if cfg.mla:  # the MLA attention output width is heads x v_dim; head_dim is not part of it
        cfg = dataclasses.replace(cfg, head_dim=cfg.hidden // cfg.heads)
    model = decode.synth_model(cfg, "som_" + which)
    write_model(tmp_path, cfg, model, n_shared=1 if cfg.shared_ffn else 0)
    got, t, m = load_decode_model(str(tmp_path))
    try:
        for f in FIELDS:
            assert getattr(got, f) == getattr(cfg, f), f
        assert abs(got.eps - cfg.eps) <= 1e-6 * cfg.eps
        for k, v in got.dtypes.items():
            assert cfg.dtypes[k] == v, k
        assert set(t) == set(model)
        for k, v in model.items():
            assert np.array_equal(np.asarray(t[k]).view(np.uint8), np.asarray(v).view(np.uint8)), k
    finally:
        m.close()


def test_refuses_what_the_engine_does_not_take(tmp_path):
    cfg = decode.TINY_MOE
    model = decode.synth_model(cfg, "som_refuse")
    write_model(tmp_path, cfg, model, n_shared=2)  # two shared experts
    with pytest.raises(SomError):
        load_decode_model(str(tmp_path))


def test_head_dim_from_the_layer_spec(tmp_path):
    """Qwen3-style attention: head_dim 128 with hidden / heads = 64.  The layer spec's
    v_head_dim gives the width (Manifest::effective_head_dim, manifest.rs:453-465), so the
    q / k / v rows come back as heads x 128 and kv_heads x 128."""
    cfg = dataclasses.replace(decode.TINY_MOE_NS, heads=8, kv_heads=2, head_dim=128)  # hidden 512 / 8 = 64
    assert cfg.q_dim != cfg.hidden
    model = decode.synth_model(cfg, "som_hd")
    write_model(tmp_path, cfg, model, v_dim=cfg.head_dim)
    got, t, m = load_decode_model(str(tmp_path))
    try:
        assert got.head_dim == 128 and got.q_dim == 1024 and got.kv_dim == 256
        assert set(t) == set(model)
    finally:
        m.close()


def test_manifest_extensions(tmp_path):
    """A version-8 manifest with YaRN (factor 16 over a 64-position original context) loads
    as the YaRN configuration; a version-7 manifest with a logit soft cap or a sliding
    window, which the engine does not apply, is refused rather than loaded as something
    else."""
    cfg = decode.TINY
    model = decode.synth_model(cfg, "som_ext")
    yarn = (16.0, 64, 32.0, 1.0)
    write_model(tmp_path, cfg, model, version=8, ext=(0.0, 0.0, 0.0, False, (), (), yarn))
    got, t, m = load_decode_model(str(tmp_path))
    m.close()
    assert got.yarn == yarn
    for i, (version, ext) in enumerate([(7, (0.0, 30.0, 0.0, False, (), (), (0.0, 0, 0.0, 0.0))),
                                        (7, (0.0, 0.0, 0.0, False, (0, 512), (), (0.0, 0, 0.0, 0.0)))]):
        d = tmp_path / f"r{i}"
        d.mkdir()
        write_model(d, cfg, model, version=version, ext=ext)
        with pytest.raises(SomError):
            load_decode_model(str(d))
