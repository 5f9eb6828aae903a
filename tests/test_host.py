"""Host-side logic of forgeserve_b200 that needs no GPU: configuration, stage split, micro-batch rows, block
allocation, stage construction and weight loading, the fused-weight views, the export list."""

import os

import pytest
import torch

import forgeserve_b200 as fs
from forgeserve_b200 import BlockAllocator, ModelConfig, OutOfBlocks, PipelineStage, bubble_fraction, stage_layers
from forgeserve_b200.kv import ContiguousKV
from forgeserve_b200.pipeline import microbatch_sizes
from oracle import forge_oracle as O


def small_cfg(**kw):
    base = dict(vocab_size=64, d_model=64, n_layers=3, n_heads=8, n_kv_heads=4, max_seq_len=64)
    base.update(kw)
    return ModelConfig(**base)


def test_export_list_matches_the_reference():
    want = ["PipelineStage", "PipelineState", "bubble_fraction", "pipeline_forward", "pipeline_generate", "stage_layers",
            "speculative_generate", "verify_draft", "Engine", "Request", "BlockAllocator", "OutOfBlocks", "PagedKVPool",
            "ModelConfig", "ForgeModel", "TPContext", "SINGLE", "ContiguousKV", "new_contiguous_cache", "generate",
            "sample"]
    assert sorted(fs.__all__) == sorted(want)
    for name in want:
        assert hasattr(fs, name)


def test_config_validation_and_defaults():
    with pytest.raises(ValueError):
        ModelConfig(d_model=100, n_heads=3)
    with pytest.raises(ValueError):
        ModelConfig(n_heads=8, n_kv_heads=3)
    with pytest.raises(ValueError):
        ModelConfig(d_model=24, n_heads=8, n_kv_heads=4)        # head_dim 3 is odd
    with pytest.raises(ValueError):
        small_cfg().check_tensor_parallel(3)
    small_cfg().check_tensor_parallel(4)
    for d in (64, 104, 136, 2048, 4096, 8192):
        assert ModelConfig(d_model=d, n_heads=4, n_kv_heads=2).ffn_dim == O.Cfg(256, d, 1, 4, 2).ffn_dim
    assert ModelConfig().to_dict()["ffn_dim"] == 384


def test_stage_layers_and_bubble():
    assert stage_layers(3, 3) == [(0, 1), (1, 2), (2, 3)]
    assert stage_layers(7, 3) == [(0, 3), (3, 5), (5, 7)]
    with pytest.raises(ValueError):
        stage_layers(2, 3)
    for n in range(1, 40):
        for p in range(1, min(n, 9) + 1):
            assert stage_layers(n, p) == O.stage_layers(n, p)
    assert bubble_fraction(1, 5) == 0
    assert bubble_fraction(4, 1) == 0.75
    assert bubble_fraction(4, 13) == pytest.approx(3 / 16)
    assert bubble_fraction(8, 16) == pytest.approx(7 / 23)


def test_microbatch_rows_follow_tensor_split():
    for b in range(0, 20):
        for m in range(1, 10):
            assert microbatch_sizes(b, m) == [len(c) for c in torch.arange(b).tensor_split(m)]


def test_allocator_order_and_errors():
    a = BlockAllocator(4)
    got = a.allocate(3)
    assert got == [0, 1, 2] and a.num_free == 1
    with pytest.raises(OutOfBlocks):
        a.allocate(2)
    a.release(got)
    assert a.num_free == 4
    assert a.allocate(2) == [2, 1]            # last released first, as the reference's stack


def test_stage_construction_and_load_from_full():
    cfg = small_cfg(n_layers=5)
    full = O.test_model_weights(O.Cfg(**{k: v for k, v in cfg.to_dict().items()}), seed=3)
    total = sum(v.numel() for k, v in full.items() if k.startswith("layers."))
    seen = 0
    for rank, size in [(0, 2), (1, 2)]:
        st = PipelineStage(cfg, rank, size, device="cpu")
        st.load_from_full(full)
        assert (st.lo, st.hi) == stage_layers(5, 2)[rank]
        assert st.is_first == (rank == 0) and st.is_last == (rank == 1)
        assert hasattr(st, "tok_emb") == st.is_first and hasattr(st, "lm_head") == st.is_last
        for j, layer in enumerate(st.layers):
            torch.testing.assert_close(layer.attn.wk.weight, full[f"layers.{st.lo + j}.attn.wk.weight"])
        seen += sum(p.numel() for p in st.layers.parameters())
    assert seen == total                       # every layer lives on exactly one stage


def test_fused_projection_weights_are_views_of_the_parameters():
    cfg = small_cfg()
    st = PipelineStage(cfg, 0, 1, device="cpu")
    full = O.test_model_weights(O.Cfg(**cfg.to_dict()), seed=4)
    st.load_from_full(full)
    blk = st.layers[1]
    wqkv = blk.attn.wqkv()
    torch.testing.assert_close(wqkv, torch.cat([full["layers.1.attn.wq.weight"], full["layers.1.attn.wk.weight"],
                                                full["layers.1.attn.wv.weight"]]))
    assert blk.attn.wq.weight.data_ptr() == wqkv.data_ptr()
    assert blk.attn.wqkv() is wqkv                       # cached while the parameters still alias it
    # loading new weights writes through the views into the fused tensor
    full2 = O.test_model_weights(O.Cfg(**cfg.to_dict()), seed=5)
    st.load_from_full(full2)
    torch.testing.assert_close(blk.attn.wqkv()[: cfg.d_model], full2["layers.1.attn.wq.weight"])
    wgu = blk.mlp.w_gate_up()
    torch.testing.assert_close(wgu[cfg.ffn_dim:], full2["layers.1.mlp.w_up.weight"])
    # the state dict keeps the reference's keys and shapes
    sd = st.state_dict()
    assert sd["layers.1.attn.wk.weight"].shape == (cfg.n_kv_heads * cfg.head_dim, cfg.d_model)
    assert "layers.1.attn._wqkv" not in sd
    # .to() replaces the parameters; the fused tensor is rebuilt from them
    st = st.to(torch.bfloat16)
    assert blk.attn.wqkv().dtype == torch.bfloat16


def test_contiguous_cache_grows_and_truncates():
    kv = ContiguousKV(max_len=10)
    k = torch.randn(2, 3, 4, 5)
    kall, _ = kv.update(k, k)
    assert kall.shape == (2, 3, 4, 5) and kv.length == 4
    kall, _ = kv.update(k[:, :, :1], k[:, :, :1])
    assert kv.length == 5 and kv.capacity <= 16
    torch.testing.assert_close(kall[:, :, :4], k)
    kv.truncate(2)
    assert kv.length == 2 and kv.k.shape[2] == 2


def test_kernels_refuse_cpu_tensors():
    from forgeserve_b200 import ops
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.rmsnorm(torch.randn(2, 8), torch.ones(8), 1e-5)
    with pytest.raises(RuntimeError, match="CUDA"):
        fs.ForgeModel(small_cfg())(torch.zeros(1, 3, dtype=torch.long))


def test_out_of_scope_names_refuse():
    with pytest.raises(NotImplementedError):
        fs.speculative_generate(None, None, None, 1)


def test_shard_state_dict_cuts_and_rebuilds_the_model():
    """forgeserve/tensor_parallel.py:25-39: q/k/v/gate/up by output rows, wo/down by input columns, the rest
    replicated; the shards put back together are the full weights; sizes that do not divide are refused."""
    from forgeserve_b200.tensor_parallel import shard_state_dict
    cfg = small_cfg()
    full = O.test_model_weights(O.Cfg(**cfg.to_dict()), seed=2)
    for size in (2, 4):
        shards = [shard_state_dict(full, cfg, r, size) for r in range(size)]
        for name, w in full.items():
            parts = [sh[name] for sh in shards]
            assert all(p.is_contiguous() for p in parts)
            if name.endswith(("wq.weight", "wk.weight", "wv.weight", "w_gate.weight", "w_up.weight")):
                assert torch.equal(torch.cat(parts, 0), w) and parts[0].shape[0] == w.shape[0] // size
            elif name.endswith(("wo.weight", "w_down.weight")):
                assert torch.equal(torch.cat(parts, 1), w) and parts[0].shape[1] == w.shape[1] // size
            else:
                assert all(torch.equal(p, w) for p in parts)
            assert all(torch.equal(p, q) for p, q in zip(parts, [O.shard(full, r, size)[name] for r in range(size)]))
    with pytest.raises(ValueError, match="n_kv_heads"):
        shard_state_dict(full, cfg, 0, 8)                    # 4 KV heads over 8 shards
    with pytest.raises(ValueError):
        fs.ForgeModel(cfg, fs.TPContext(0, 8))


def test_tensor_parallel_model_holds_its_shard():
    """ForgeModel(cfg, TPContext(rank, size)): a shard's heads and hidden features, the reference's keys, and a
    shard of the state dict loads into it (the replicated embedding stays tied to the head)."""
    from forgeserve_b200.tensor_parallel import shard_state_dict
    cfg = small_cfg()
    full = O.test_model_weights(O.Cfg(**cfg.to_dict()), seed=2)
    m = fs.ForgeModel(cfg, fs.TPContext(1, 2), device="cpu")
    a, mlp = m.layers[0].attn, m.layers[0].mlp
    assert (a.nh, a.nkv, a.hd) == (4, 2, 8)
    assert a.wq.weight.shape == (32, 64) and a.wk.weight.shape == (16, 64) and a.wo.weight.shape == (64, 32)
    assert mlp.w_gate.weight.shape == (cfg.ffn_dim // 2, 64) and mlp.w_down.weight.shape == (64, cfg.ffn_dim // 2)
    m.load_state_dict(shard_state_dict(full, cfg, 1, 2))
    assert torch.equal(a.wqkv()[:32], full["layers.0.attn.wq.weight"][32:])
    assert m.lm_head.weight is m.tok_emb.weight
    pool = fs.PagedKVPool(cfg, 8, 4, tp=m.tp)
    assert pool.k[0].shape == (8, 2, 4, 8)


def _mapped_ranges(path):
    """Address ranges of this process's mappings of `path` (Linux /proc/self/maps)."""
    real = os.path.realpath(path)
    out = []
    with open("/proc/self/maps") as f:
        for line in f:
            parts = line.split()
            if len(parts) >= 6 and parts[5] == real:
                lo, hi = (int(x, 16) for x in parts[0].split("-"))
                out.append((lo, hi))
    return out


def test_stages_load_from_a_mapped_state_dict_file(tmp_path):
    """Per-stage loading from the reference's saved format (torch.save of the state dict, tied head): the file is
    mapped, not read, and each stage ends up with the same weights as load_from_full of the in-memory dict."""
    from forgeserve_b200.weights import open_state_dict
    cfg = small_cfg(n_layers=5)
    full = O.test_model_weights(O.Cfg(**cfg.to_dict()), seed=6)
    assert full["lm_head.weight"] is full["tok_emb.weight"]
    path = tmp_path / "model.pt"
    torch.save(full, path)
    mapped = open_state_dict(path)
    assert set(mapped) == set(full)
    ranges = _mapped_ranges(path)
    assert ranges, "the state dict file is not memory-mapped"
    for k, t in mapped.items():
        assert any(lo <= t.data_ptr() < hi for lo, hi in ranges), k      # a view of the file, not a host copy
    assert mapped["lm_head.weight"].data_ptr() == mapped["tok_emb.weight"].data_ptr()
    for rank in range(3):
        a = PipelineStage(cfg, rank, 3, device="cpu")
        a.load_from_file(path)
        b = PipelineStage(cfg, rank, 3, device="cpu")
        b.load_from_full(full)
        sa, sb = a.state_dict(), b.state_dict()
        assert set(sa) == set(sb)
        for k in sa:
            assert torch.equal(sa[k], sb[k]), (rank, k)
    # a stage built in bf16 takes the fp32 file's tensors rounded, as load_from_full does
    c = PipelineStage(cfg, 1, 3, device="cpu", dtype=torch.bfloat16)
    c.load_from_file(path)
    lo = c.lo
    assert torch.equal(c.layers[0].mlp.w_down.weight, full[f"layers.{lo}.mlp.w_down.weight"].to(torch.bfloat16))


def test_tensor_parallel_stage_needs_the_grid_transport():
    with pytest.raises(ValueError, match="make_grid"):
        PipelineStage(small_cfg(), 0, 2, device="cpu", tp=fs.TPContext(0, 2))


def test_seeded_weights_of_tensor_parallel_shards():
    """weights.init_stage_ / init_model_ on tensor-parallel modules: each shard holds its cut of the same seeded
    tensors that a whole stage or model gets."""
    from forgeserve_b200.tensor_parallel import shard_state_dict
    from forgeserve_b200.weights import init_model_, init_stage_, seeded_state_dict
    cfg = small_cfg()
    full = seeded_state_dict(cfg, seed=3)
    for rank in range(2):
        # the stages only hold weights here: a placeholder stands in for the grid transport
        st = PipelineStage(cfg, 1, 2, device="cpu", tp=fs.TPContext(rank, 2), transport=object())
        init_stage_(st, seed=3)
        want = PipelineStage(cfg, 1, 2, device="cpu", tp=fs.TPContext(rank, 2), transport=object())
        want.load_from_full(full)
        for (k, a), (_, b) in zip(st.state_dict().items(), want.state_dict().items()):
            assert torch.equal(a, b), k
        m = fs.ForgeModel(cfg, fs.TPContext(rank, 2), device="cpu")
        init_model_(m, seed=3)
        shard = shard_state_dict(full, cfg, rank, 2)
        for k, v in m.state_dict().items():
            assert torch.equal(v, shard[k]), k
