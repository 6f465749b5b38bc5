"""Host-side logic on CPU: asset loading, parameters, errors, plugin registration,
the vLLM hooks and the buffer derivation used by the kernels."""

from __future__ import annotations

import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import PKG, REPO


@pytest.fixture(scope="module")
def small_assets(tmp_path_factory, golden_small):
    """The small golden head written in the reference's asset layout."""
    from flash_head.synthetic import HeadShape, SyntheticHead, save_assets
    g = golden_small
    W = torch.from_numpy(g["weight_bits"].view(np.int16)).view(torch.bfloat16)
    head = SyntheticHead(weight=W, centroids=torch.from_numpy(g["centroids"]),
                         assignments=torch.from_numpy(g["assignments"]),
                         shape=HeadShape(hidden=64, vocab=2048, n_clusters=128, n_probes=8),
                         seed=11)
    d = str(tmp_path_factory.mktemp("model"))
    save_assets(head, d, n_probes=8, special_token_ids=[0, 7, 2047])
    return d, head


def test_metadata_and_weight_loading(small_assets):
    from flash_head import loading
    d, head = small_assets
    meta = loading.load_flash_head_from_checkpoint(d)
    assert meta["cache_dir"] == os.path.join(d, "flash_head_assets")
    assert meta["special_token_ids"] == [0, 7, 2047] and meta["n_probes"] == 8
    w, key = loading.lm_head_weight(loading.ModelFiles(d))
    assert key == "lm_head.weight" and torch.equal(w, head.weight)
    assert loading.load_flash_head_from_checkpoint(os.path.join(d, "missing")) is None


def test_sharded_index_and_tied_embedding(tmp_path):
    from safetensors.torch import save_file

    from flash_head import assets
    w = torch.randn(32, 8)
    save_file({"model.embed_tokens.weight": w}, str(tmp_path / "shard-1.safetensors"))
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps(
        {"weight_map": {"model.embed_tokens.weight": "shard-1.safetensors",
                        "model.layers.0.w": "shard-2.safetensors"}}))
    got, key = assets.lm_head_weight(assets.ModelFiles(str(tmp_path)))
    assert key == "model.embed_tokens.weight" and torch.equal(got, w)
    # an index may name the head under any prefix; a single file only by LM_HEAD_KEYS
    assert assets.pick_lm_head_key(["x.lm_head.weight"], by_suffix=True) == "x.lm_head.weight"
    assert assets.pick_lm_head_key(["x.lm_head.weight"], by_suffix=False) is None
    assert assets.pick_lm_head_key(["model.embed_tokens.weight", "lm_head.weight"],
                                   by_suffix=True) == "lm_head.weight"
    with pytest.raises(FileNotFoundError, match="No supported weight files"):
        assets.lm_head_weight(assets.ModelFiles(str(tmp_path / "nothing")))


def test_parameters_match_the_reference_layout(small_assets, golden_small):
    from flash_head.flash_head import FlashHead, get_flash_head_parameters
    d, head = small_assets
    lm = torch.nn.Linear(64, 2048, bias=False)
    lm.weight.data.copy_(head.weight.float())
    params = get_flash_head_parameters(lm, os.path.join(d, "flash_head_assets"), d)
    assert np.array_equal(params["vocab_maps_tensor"].numpy(), golden_small["ref_vocab_maps"])
    fh = FlashHead(lm, **params, n_probes=8, special_token_ids=[0, 7]).to(dtype=torch.bfloat16)
    cw_bits = fh.cluster_linear.weight.detach().contiguous().view(torch.int16).numpy()
    assert np.array_equal(cw_bits.view(np.uint16), golden_small["ref_cluster_w_bits"])
    vm = params["vocab_maps_tensor"]
    assert torch.equal(fh.w_perm.view(-1, 64), head.weight[vm.reshape(-1)])
    assert fh.n_probes == 8 and fh.special_token_ids_tensor.tolist() == [0, 7]
    # no CPU fallback for the step itself
    with pytest.raises(RuntimeError, match="CUDA"):
        fh.get_next_token(torch.zeros(1, 1, 64, dtype=torch.bfloat16))


def test_errors_match_the_reference():
    from flash_head.flash_head import FlashHead, vocab_maps_from_assignments
    with pytest.raises(ValueError, match="balanced"):
        vocab_maps_from_assignments(torch.tensor([0, 0, 1]), 2)
    lm = torch.nn.Linear(16, 32, bias=False)
    vm = torch.arange(32).view(2, 16)
    missing = vm.clone()
    missing[1, 15] = 0  # vocab id 31 appears nowhere
    with pytest.raises(ValueError, match="missing from vocab_maps"):
        FlashHead(lm, torch.randn(16, 2), missing, special_token_ids=[31])
    with pytest.raises(AssertionError, match="unbalanced"):
        FlashHead(lm, torch.randn(16, 2), vm[:, :8])
    assert FlashHead(lm, torch.randn(16, 2), vm).n_probes == 0  # K / 16, as the reference


def test_broken_cache_is_a_value_error(tmp_path, small_assets):
    from safetensors.torch import save_file

    from flash_head.flash_head import _get_centroids
    d, _ = small_assets
    bad = tmp_path / "c"
    bad.mkdir()
    save_file({"centroids": torch.zeros(64, 128)}, str(bad / "clustering_cache.safetensors"))
    lm = torch.nn.Linear(64, 2048, bias=False)
    with pytest.raises(ValueError, match="Error loading cache"):
        _get_centroids(lm, str(tmp_path), "c")


def test_derive_and_shard_buffers(golden_small):
    from flash_head.native import derive_buffers, quantize_rows_fp8, shard_buffers
    from flash_head.tp import cluster_range
    g = golden_small
    W = torch.from_numpy(g["weight_bits"].view(np.int16)).view(torch.bfloat16)
    vm = torch.from_numpy(g["ref_vocab_maps"])
    w_perm = W[vm.reshape(-1)].view(128, 16, 64)
    cw = torch.from_numpy(O_norm(g["centroids"]))
    bufs = derive_buffers(w_perm, vm, cw, torch.from_numpy(g["centroids"]),
                          torch.tensor([7, 2047]), "fp8")
    assert bufs["cluster_w"].dtype == torch.float8_e4m3fn
    deq = bufs["cluster_w"].float() * bufs["cluster_scale"][:, None]
    assert torch.allclose(deq, cw.bfloat16().float(), rtol=0.07, atol=1e-6)
    q, sc = quantize_rows_fp8(torch.zeros(2, 16))
    assert torch.isfinite(sc).all() and (q.float() == 0).all()
    flat = vm.reshape(-1)
    assert [int(flat[s]) for s in bufs["special_slots"]] == [7, 2047]
    parts = [shard_buffers(bufs, 16, *cluster_range(128, 3, r)) for r in range(3)]
    assert torch.equal(torch.cat([p["w_perm"] for p in parts]), bufs["w_perm"])
    assert torch.equal(torch.cat([p["vocab_map"] for p in parts]), bufs["vocab_map"])
    rebased = [(r, int(s)) for r, p in enumerate(parts) if p["special_slots"] is not None
               for s in p["special_slots"]]
    assert len(rebased) == 2
    for r, s in rebased:
        lo, _ = cluster_range(128, 3, r)
        assert int(bufs["vocab_map"][lo * 16 + s]) in (7, 2047)


def test_derive_buffers_of_a_shard_slice(golden_small):
    """A tensor-parallel shard derives its buffers from its clusters alone,
    whose vocab ids are a subset of the vocabulary, not a permutation of
    [0, K_shard * cap)."""
    from flash_head.native import derive_buffers
    g = golden_small
    W = torch.from_numpy(g["weight_bits"].view(np.int16)).view(torch.bfloat16)
    vm = torch.from_numpy(g["ref_vocab_maps"])
    w_perm = W[vm.reshape(-1)].view(128, 16, 64)
    cw = torch.from_numpy(O_norm(g["centroids"]))
    craw = torch.from_numpy(g["centroids"])
    sl = slice(64, 128)
    part = derive_buffers(w_perm[sl], vm[sl], cw[sl], craw[:, sl], torch.zeros(0, dtype=torch.int64),
                          "fp8")
    assert part["special_slots"] is None and part["w_perm"].shape == (64 * 16, 64)
    inside = int(vm[100, 3])
    part = derive_buffers(w_perm[sl], vm[sl], cw[sl], craw[:, sl], torch.tensor([inside]), "fp8")
    assert part["special_slots"].tolist() == [(100 - 64) * 16 + 3]
    with pytest.raises(ValueError, match="missing"):
        derive_buffers(w_perm[sl], vm[sl], cw[sl], craw[:, sl], torch.tensor([int(vm[3, 0])]), "fp8")


def O_norm(centroids):
    from oracle import flashhead_oracle as O
    return O.normalized_cluster_weight(centroids)


def test_cluster_ranges_partition():
    from flash_head.tp import cluster_range
    for K in (7, 8016, 9496):
        for R in (1, 2, 3, 8):
            rs = [cluster_range(K, R, r) for r in range(R)]
            assert rs[0][0] == 0 and rs[-1][1] == K
            assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
    with pytest.raises(ValueError):
        cluster_range(10, 2, 2)


_REGISTER_SCRIPT = r"""
import os, sys
sys.path.insert(0, {pkg!r})
os.environ["FLASHHEAD_ENABLED"] = {enabled!r}
import flash_head
from vllm.model_executor.layers.logits_processor import LogitsProcessor
from vllm.v1.sample.sampler import Sampler
from vllm.v1.worker.gpu_model_runner import GPUModelRunner
seen = {{}}
def fake_dummy_sampler_run(self, h):  # stands in for vLLM's warm-up (no GPU here)
    from flash_head.patches import logits_processor as lp
    seen["ids_inside"] = lp.flash_head_token_ids(h)
    return "vllm-warmup"
GPUModelRunner._dummy_sampler_run = fake_dummy_sampler_run
before = (LogitsProcessor._get_logits, Sampler.forward)
flash_head.register(); flash_head.register()
after = (LogitsProcessor._get_logits, Sampler.forward)
from vllm import ModelRegistry
archs = ModelRegistry.get_supported_archs()
print("PATCHED" if after != before else "UNPATCHED", "FlashHeadLlamaForCausalLM" in archs)
if after != before:
    import torch
    from flash_head.patches import logits_processor as lp
    class FakeHead:
        def get_next_token_batched(self, h):
            return torch.arange(h.shape[0], dtype=torch.int64) + 5
    class CountingHead(FakeHead):
        calls = 0
        def get_next_token_batched(self, h):
            CountingHead.calls += 1
            return super().get_next_token_batched(h)
    lp._flash_head = CountingHead()
    r = GPUModelRunner._dummy_sampler_run(None, torch.zeros(3, 8))
    print("WARMUP", r, seen["ids_inside"], CountingHead.calls)
    import tempfile
    from flash_head.synthetic import HeadShape, make_head, save_assets
    from flash_head.loading import METADATA_PATH
    from flash_head.patches import engine
    from vllm.v1.engine.llm_engine import LLMEngine
    d = tempfile.mkdtemp()
    save_assets(make_head(HeadShape(hidden=16, vocab=64, n_clusters=4, n_probes=2), seed=1), d)
    print("ENGINE", hasattr(LLMEngine.from_engine_args, "__wrapped__"),
          engine.publish_metadata(d), os.path.exists(METADATA_PATH),
          engine.publish_metadata(tempfile.mkdtemp()), os.path.exists(METADATA_PATH))
    lp._flash_head = FakeHead()
    proc = LogitsProcessor.__new__(LogitsProcessor)
    proc.logits_as_input = False; proc.soft_cap = 30.0; proc.scale = 2.0
    ids = proc.forward(None, torch.zeros(1, 8))
    print("IDS", ids.dtype, ids.tolist())
    out = Sampler.forward(Sampler.__new__(Sampler), ids, None)
    print("SAMPLED", out.sampled_token_ids.tolist(), out.logprobs_tensors)
    from types import SimpleNamespace
    class FakeHeadLogprobs(FakeHead):
        def candidate_logprobs(self, h, tok, k):
            n = h.shape[0]
            print("ASKED", tok.tolist(), k, tuple(h.shape))
            return (torch.full((n, k + 1), 7, dtype=torch.int32), torch.zeros(n, k + 1),
                    torch.ones(n, dtype=torch.int64))
    lp._flash_head = FakeHeadLogprobs()
    ids = proc.forward(None, torch.zeros(1, 8))
    md = SimpleNamespace(max_num_logprobs=3, logprob_token_ids=None)
    t = Sampler.forward(Sampler.__new__(Sampler), ids, md).logprobs_tensors
    print("LOGPROBS", type(t).__name__, tuple(t.logprob_token_ids.shape), t.logprob_token_ids.dtype,
          tuple(t.logprobs.shape), t.selected_token_ranks.tolist())
    # speculative decoding: verification of drafts against FlashHead ids (the
    # device comparison replaced by the oracle here: no GPU on this path)
    import numpy as np
    from oracle import flashhead_oracle as O
    import flash_head.spec as spec
    def fake_accept(draft, target, bonus, cu, max_spec_len, placeholder=-1, out=None):
        cu = cu.tolist()
        num = [c - (cu[i - 1] if i else 0) for i, c in enumerate(cu)]
        return torch.from_numpy(O.spec_accept(draft.numpy(), target.numpy(), bonus.numpy(),
                                              num, max_spec_len, placeholder))
    spec.accept_draft_tokens = fake_accept
    from vllm.v1.sample.rejection_sampler import RejectionSampler
    from vllm.v1.spec_decode.metadata import SpecDecodeMetadata
    md = SpecDecodeMetadata.make_dummy([[5, 6], [7], []], device="cpu")
    md.target_logits_indices = torch.tensor([0, 1, 3], dtype=torch.int32)
    md.bonus_logits_indices = torch.tensor([2, 4, 5], dtype=torch.int32)
    step_ids = torch.tensor([[5], [6], [30], [8], [31], [32]], dtype=torch.int32)
    rs = RejectionSampler.__new__(RejectionSampler)
    print("SPEC", RejectionSampler.forward(rs, md, None, step_ids, None).sampled_token_ids.tolist())
    from vllm.v1.spec_decode.eagle import EagleProposer
    prop = EagleProposer.__new__(EagleProposer)
    prop.use_local_argmax_reduction = False
    prop.model = SimpleNamespace(compute_logits=lambda h: torch.tensor([[11], [12]], dtype=torch.int32))
    print("DRAFT", prop._greedy_sample(torch.zeros(2, 8)).tolist(),
          prop._sample_from_logits(torch.tensor([[3]], dtype=torch.int32), None)[0].tolist())
    for bad in (SimpleNamespace(max_num_logprobs=-1, logprob_token_ids=None),
                SimpleNamespace(max_num_logprobs=2, logprob_token_ids={{0: [3]}})):
        print("UNSUPPORTED", Sampler.forward(Sampler.__new__(Sampler), ids, bad).logprobs_tensors)
    # per-request temperature: greedy rows keep the greedy ids, the others are
    # sampled once per distinct temperature, seeded from a request's generator
    calls = []
    class FakeHeadSample(FakeHead):
        def get_next_token_batched(self, h, do_sample=False, temperature=1.0, seed=0, offset=0):
            if not do_sample:
                return super().get_next_token_batched(h)
            calls.append((h.shape[0], round(temperature, 3), seed))
            return torch.full((h.shape[0],), int(round(temperature * 100)), dtype=torch.int64)
    lp._flash_head = FakeHeadSample()
    lp.max_decode_rows = lambda: 4
    ids = proc.forward(None, torch.zeros(4, 8))
    md = SimpleNamespace(max_num_logprobs=None, logprob_token_ids=None, all_greedy=False,
                         temperature=torch.tensor([0.0, 0.7, 0.7, 1.3]), top_k=None, top_p=None,
                         generators={{2: torch.Generator().manual_seed(3)}})
    out = Sampler.forward(Sampler.__new__(Sampler), ids, md)
    want_seed = int(torch.randint(0, 2**62, (1,), generator=torch.Generator().manual_seed(3)).item())
    print("TEMPERATURE", out.sampled_token_ids.view(-1).tolist(), [c[:2] for c in calls],
          calls[0][2] == want_seed)
"""


@pytest.mark.parametrize("enabled", ["1", "0"])
def test_register_and_hooks(enabled):
    pytest.importorskip("vllm")
    code = _REGISTER_SCRIPT.format(pkg=PKG, enabled=enabled)
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=600, cwd=REPO)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = res.stdout.strip().splitlines()
    status = [ln for ln in lines if ln.startswith(("PATCHED", "UNPATCHED"))][0]
    assert status.split()[1] == "True"  # architecture aliases registered either way
    if enabled == "1":
        assert status.startswith("PATCHED")
        # warm-up: one FlashHead step, vLLM's own warm-up on real logits
        assert "WARMUP vllm-warmup None 1" in res.stdout
        # engine hooks: metadata published for a FlashHead model, withdrawn for another
        assert "ENGINE True True True False False" in res.stdout
        assert "IDS torch.int32 [[5]]" in res.stdout  # ids untouched by soft-cap / scale
        assert "SAMPLED [[5]] None" in res.stdout
        # logprobs over the step's candidate set when a request asks for k of them
        assert "ASKED [5] 3 (1, 8)" in res.stdout
        assert "LOGPROBS LogprobsTensors (1, 4) torch.int32 (1, 4) [1]" in res.stdout
        assert res.stdout.count("UNSUPPORTED None") == 2
        # drafts [5, 6] vs targets [5, 6] -> bonus 30; [7] vs [8] -> 8; no drafts -> bonus 32
        assert "SPEC [[5, 6, 30], [8, -1, -1], [32, -1, -1]]" in res.stdout
        assert "DRAFT [11, 12] [3]" in res.stdout
        assert "TEMPERATURE [5, 70, 70, 130] [(2, 0.7), (1, 1.3)] True" in res.stdout
    else:
        assert status.startswith("UNPATCHED")
