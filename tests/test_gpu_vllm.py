"""vLLM end to end: a model served by vLLM decodes through this FlashHead.

A tiny Llama (2 layers, hidden 512, vocabulary 4096 = 256 balanced clusters
of 16) is written in the reference's asset layout: ``FlashHeadLlamaForCausalLM``
architecture, ``flash_head_cache_dir`` and ``n_probes`` in config.json, the
clustering cache beside it (loading.py:179-205, flash_head.py:41-78). Its LM
head is a seeded centre+noise head, the other weights are random.

vLLM 0.22 runs in a child process that finds the plugin the way an installed
package is found: through a ``vllm.general_plugins`` entry point
(``flash_head = flash_head:register``) of a distribution on the path. The
engine runs in-process (VLLM_ENABLE_V1_MULTIPROCESSING=0) so the child can
count the FlashHead steps of its worker.

Checked:
  * greedy generation goes through the FlashHead hook (every decode step of
    one row returns FlashHead token ids), and each generated token is the
    oracle's FlashHead greedy token for the hidden state a reference forward
    pass (transformers, fp32) computes on the same prefix, or a logit
    near-tie of it (vLLM computes the hidden states in bf16);
  * with FLASHHEAD_MAX_DECODE_ROWS=4, three concurrent requests decode
    through FlashHead's batched step with the same per-token check;
  * a request for logprobs gets FlashHead's candidate-set logprobs, with the
    sampled token's among them;
  * a request with a temperature and a seed is sampled by FlashHead's
    sampling kernels, reproducibly.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import PKG, REPO
from oracle import flashhead_oracle as O

pytestmark = pytest.mark.gpu

D, V, K, P = 512, 4096, 256, 16


def _write_model(d: str):
    from safetensors.torch import save_file
    from transformers import LlamaConfig, LlamaForCausalLM

    from flash_head.synthetic import HeadShape, make_head
    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=D, intermediate_size=1024, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=8, vocab_size=V,
                      max_position_embeddings=512, rms_norm_eps=1e-5, rope_theta=10000.0,
                      tie_word_embeddings=False, bos_token_id=1, eos_token_id=2)
    model = LlamaForCausalLM(cfg).to(torch.bfloat16)
    head = make_head(HeadShape(hidden=D, vocab=V, n_clusters=K, n_probes=P), seed=3)
    with torch.no_grad():
        model.lm_head.weight.copy_(head.weight)
        model.model.embed_tokens.weight.mul_(20.0)  # hidden states of a usable scale
    model.save_pretrained(d)
    os.makedirs(os.path.join(d, "flash_head_assets"), exist_ok=True)
    save_file({"centroids": head.centroids.contiguous(),
               "cluster_assignments": head.assignments.contiguous()},
              os.path.join(d, "flash_head_assets", "clustering_cache.safetensors"))
    with open(os.path.join(d, "config.json")) as f:
        conf = json.load(f)
    conf["architectures"] = ["FlashHeadLlamaForCausalLM"]
    conf["flash_head_cache_dir"] = "flash_head_assets"
    conf["n_probes"] = P
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(conf, f)
    return head


def _plugin_site(d: str) -> str:
    """A distribution that declares the plugin's entry point, as pip would."""
    site = os.path.join(d, "site")
    info = os.path.join(site, "flash_head_b200-0.1.10.dist-info")
    os.makedirs(info, exist_ok=True)
    with open(os.path.join(info, "METADATA"), "w") as f:
        f.write("Metadata-Version: 2.1\nName: flash-head-b200\nVersion: 0.1.10\n")
    with open(os.path.join(info, "entry_points.txt"), "w") as f:
        f.write("[vllm.general_plugins]\nflash_head = flash_head:register\n")
    return site


_DRIVER = r"""
import json, os, sys
from vllm import LLM, SamplingParams
model, prompts, max_tokens, logprobs = sys.argv[1], json.loads(sys.argv[2]), int(sys.argv[3]), int(sys.argv[4])
temperature, seed = float(sys.argv[5]), int(sys.argv[6])
llm = LLM(model=model, skip_tokenizer_init=True, enforce_eager=True, dtype="bfloat16",
          gpu_memory_utilization=0.25, max_model_len=256, max_num_seqs=8, seed=0)
from flash_head.patches import logits_processor as lp
steps = []
inner = lp.flash_head_token_ids
def counted(h):
    ids = inner(h)
    steps.append((int(h.shape[0]), ids is not None))
    return ids
lp.flash_head_token_ids = counted
sampled = []
inner_s = lp.step_sampled_ids
def counted_s(ids, md):
    out = inner_s(ids, md)
    sampled.append(int(md is not None and not md.all_greedy))
    return out
lp.step_sampled_ids = counted_s
sp = SamplingParams(max_tokens=max_tokens, temperature=temperature, logprobs=logprobs or None,
                    ignore_eos=True, detokenize=False, seed=seed if seed >= 0 else None)
outs = llm.generate([{"prompt_token_ids": p} for p in prompts], sp)
res = {"tokens": [list(o.outputs[0].token_ids) for o in outs], "steps": steps, "sampled": sampled,
       "logprobs": [[{str(k): float(v.logprob) for k, v in pos.items()} for pos in (o.outputs[0].logprobs or [])]
                    for o in outs]}
print("RESULT " + json.dumps(res), flush=True)
"""


def _run_vllm(model_dir, site, prompts, max_tokens, logprobs=0, max_rows=1, temperature=0.0,
              seed=-1):
    env = dict(os.environ)
    env.update(PYTHONPATH=os.pathsep.join([site, PKG, REPO, env.get("PYTHONPATH", "")]),
               VLLM_ENABLE_V1_MULTIPROCESSING="0",
               FLASHHEAD_MAX_DECODE_ROWS=str(max_rows), TOKENIZERS_PARALLELISM="false")
    res = subprocess.run([sys.executable, "-c", _DRIVER, model_dir, json.dumps(prompts),
                          str(max_tokens), str(logprobs), str(temperature), str(seed)],
                         capture_output=True, text=True, timeout=900, env=env, cwd=model_dir)
    line = [ln for ln in res.stdout.splitlines() if ln.startswith("RESULT ")]
    assert res.returncode == 0 and line, (res.stdout[-3000:], res.stderr[-6000:])
    return json.loads(line[0][len("RESULT "):])


class _OracleHead:
    """The oracle's FlashHead greedy token (bf16 stage 1, the default) from
    final hidden states, and dense logits for the near-tie check."""

    def __init__(self, head):
        self.W = head.weight.float().numpy()
        self.vm = O.vocab_maps_from_assignments(head.assignments.numpy(), K)
        self.w_perm = O.permute_weight(self.W, self.vm)
        self.cw = O.bf16_round(O.normalized_cluster_weight(head.centroids.float().numpy()))

    def token(self, h):
        return O.greedy_token(h, self.w_perm, self.vm, self.cw, P)[0]

    def logit(self, h, v):
        return float(self.W[v].astype(np.float64) @ h.astype(np.float64))


def _check_tokens(model_dir, oracle, prompts, generated):
    """Every generated token against the oracle on the reference forward's
    hidden state of its prefix; returns the fraction of exact matches."""
    from transformers import LlamaForCausalLM
    ref = LlamaForCausalLM.from_pretrained(model_dir, torch_dtype=torch.float32).eval()
    exact = total = 0
    for prompt, toks in zip(prompts, generated):
        seq = list(prompt) + list(toks)
        with torch.no_grad():
            hs = ref.model(torch.tensor([seq])).last_hidden_state[0].numpy()
        for i, t in enumerate(toks):
            h = hs[len(prompt) + i - 1]
            want = oracle.token(h)
            total += 1
            if t == want:
                exact += 1
                continue
            a, b = oracle.logit(h, t), oracle.logit(h, want)
            assert abs(a - b) <= 2e-2 * max(abs(a), abs(b)), (prompt, i, t, want, a, b)
    return exact / total


@pytest.fixture(scope="module")
def served(tmp_path_factory):
    pytest.importorskip("vllm")
    pytest.importorskip("transformers")
    d = str(tmp_path_factory.mktemp("tiny_llama"))
    head = _write_model(d)
    return d, _plugin_site(str(tmp_path_factory.mktemp("plugin"))), _OracleHead(head)


def test_vllm_greedy_decodes_through_flashhead(served):
    model_dir, site, oracle = served
    prompts = [[1, 17, 305, 2201, 44]]
    out = _run_vllm(model_dir, site, prompts, max_tokens=12)
    assert len(out["tokens"][0]) == 12
    one_row = [used for rows, used in out["steps"] if rows == 1]
    # prefill's last position and every decode step: one row each, all FlashHead
    assert len(one_row) >= 12 and all(one_row), out["steps"]
    assert _check_tokens(model_dir, oracle, prompts, out["tokens"]) >= 0.75


def test_vllm_batched_decode_and_logprobs(served):
    model_dir, site, oracle = served
    prompts = [[1, 9, 88, 731], [1, 4000, 12], [1, 55, 56, 57, 58, 59]]
    out = _run_vllm(model_dir, site, prompts, max_tokens=8, logprobs=2, max_rows=4)
    batched = [used for rows, used in out["steps"] if rows > 1]
    assert batched and all(batched), out["steps"]  # multi-row decode steps through FlashHead
    assert _check_tokens(model_dir, oracle, prompts, out["tokens"]) >= 0.75
    for toks, lps in zip(out["tokens"], out["logprobs"]):
        assert len(lps) == len(toks)
        for t, pos in zip(toks, lps):
            vals = {int(k): v for k, v in pos.items()}
            assert t in vals and all(np.isfinite(v) and v <= 1e-6 for v in vals.values())
            assert vals[t] >= max(vals.values()) - 1e-3  # greedy: the top candidate


def test_vllm_temperature_is_sampled_by_flashhead(served):
    """A request with a temperature and a seed is sampled by FlashHead's
    sampling kernels (not decoded greedily), and the seed repeats it."""
    model_dir, site, oracle = served
    prompts = [[1, 17, 305, 2201, 44]]
    runs = [_run_vllm(model_dir, site, prompts, max_tokens=16, temperature=1.5, seed=7)
            for _ in range(2)]
    for out in runs:
        assert len(out["tokens"][0]) == 16 and all(0 <= t < V for t in out["tokens"][0])
        assert out["sampled"] and all(out["sampled"]), out["sampled"]
        assert all(used for rows, used in out["steps"] if rows == 1)
    assert runs[0]["tokens"] == runs[1]["tokens"]
    greedy = _run_vllm(model_dir, site, prompts, max_tokens=16)
    assert not any(greedy["sampled"])
