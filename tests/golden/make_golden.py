"""Generate the golden vectors that pin the oracle to the reference.

Runs the reference FlashHead (embedl/flash-head, imported from its source
tree) on CPU and records its outputs on seeded synthetic heads. It needs the
reference source, so it runs only where that tree exists; the outputs are
committed next to this script and the tests read only those files.

The reference head is built the way its vLLM loader builds it: the assets are
written in the ``flash_head_cache_dir`` layout, ``load_flash_head_from_checkpoint``
(loading.py:179-205) reads config.json, ``_load_lm_head_weight`` (:66-106)
reads the weight, ``get_flash_head_parameters`` (flash_head.py:81-118)
derives the clustering, and the module is cast to bf16 (loading.py:152-164),
on CPU instead of CUDA.

Usage:  python tests/golden/make_golden.py [--reference-src DIR] [--only NAME]

The reference source tree (the directory holding its ``flash_head`` package)
comes from ``--reference-src`` or the ``FLASHHEAD_REFERENCE_SRC`` environment
variable.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _load_synthetic():
    """Load the synthetic-head module by path: the reference package is also
    called ``flash_head``, so this repository's package must not be imported
    under that name in this process."""
    import importlib.util
    path = os.path.join(REPO, "flash-head_b200", "flash_head", "synthetic.py")
    spec = importlib.util.spec_from_file_location("fh_b200_synthetic", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


_syn = _load_synthetic()
HeadShape, LLAMA32_1B, LLAMA31_8B, QWEN25_15B = (_syn.HeadShape, _syn.LLAMA32_1B,
                                                 _syn.LLAMA31_8B, _syn.QWEN25_15B)
head_checksum, make_head, make_hidden, save_assets = (
    _syn.head_checksum, _syn.make_head, _syn.make_hidden, _syn.save_assets)

SMALL = HeadShape(hidden=64, vocab=2048, n_clusters=128, n_probes=8)
SMALL_SPECIALS = [0, 7, 2047]


def _import_reference(src: str):
    sys.path.insert(0, src)
    import flash_head.flash_head as ref_fh  # noqa: F401
    import flash_head.loading as ref_loading
    assert os.path.abspath(ref_fh.__file__).startswith(os.path.abspath(src)), ref_fh.__file__
    return ref_fh, ref_loading


def _reference_head(ref_fh, ref_loading, head, n_probes, specials):
    """Build the reference FlashHead from on-disk assets (CPU, bf16)."""
    with tempfile.TemporaryDirectory() as d:
        save_assets(head, d, n_probes=n_probes, special_token_ids=specials)
        meta = ref_loading.load_flash_head_from_checkpoint(d)
        w, _ = ref_loading._load_lm_head_weight(meta["model_path"])
        V, D = w.shape
        lm = torch.nn.Linear(D, V, bias=False)
        lm.weight.data.copy_(w)
        params = ref_fh.get_flash_head_parameters(lm, cache_dir=meta["cache_dir"],
                                                  model_or_dir=meta["model_path"])
        fh = ref_fh.FlashHead(lm, **params, n_probes=meta["n_probes"],
                              special_token_ids=meta["special_token_ids"]).to(dtype=torch.bfloat16)
    return fh


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _reference_greedy(fh, x):
    """The reference's greedy answer for one row, computed by its own code.

    Its default greedy branch is the Triton kernel (GPU only); its
    gather-and-argmax branch (flash_head.py:323-334) with
    use_identical_tiebreak=False is the same computation in torch and runs on
    CPU. (With use_identical_tiebreak=True that branch applies ``mapping`` to
    an index into the already-sorted ``indices`` (:331-333) and returns a
    token that is not the argmax; those outputs are kept as ref_tok_tiebreak.)
    """
    top = fh._get_top_clusters(x)
    logits, _, indices = fh._gather_cluster_logits(x, top, False)
    idx = logits.argmax(dim=-1, keepdim=True)
    return int(indices[idx][0].view(-1)[0])


def small_greedy(ref_fh, ref_loading, out):
    head = make_head(SMALL, seed=11)
    rows = 48
    h = make_hidden(rows, SMALL.hidden, seed=12)
    fh = _reference_head(ref_fh, ref_loading, head, SMALL.n_probes, None)
    fh_sp = _reference_head(ref_fh, ref_loading, head, SMALL.n_probes, SMALL_SPECIALS)
    sims, probes, tok_tb, tok_sp, tok_g = [], [], [], [], []
    with torch.no_grad():
        for r in range(rows):
            x = h[r].view(1, 1, -1)
            sims.append(_bits(fh.cluster_linear(x).view(-1)))
            probes.append(np.sort(fh._get_top_clusters(x).view(-1).numpy()))
            tok_g.append(_reference_greedy(fh, x))
            tok_tb.append(int(fh.get_next_token(x, use_identical_tiebreak=True).view(-1)[0]))
            tok_sp.append(int(fh_sp.get_next_token(x).view(-1)[0]))
        dense = fh.get_next_token(h.view(rows, 1, -1)).view(-1).numpy()
    np.savez_compressed(
        os.path.join(out, "small_greedy.npz"),
        weight_bits=_bits(head.weight), centroids=head.centroids.numpy(),
        assignments=head.assignments.numpy(), hidden_bits=_bits(h),
        n_probes=SMALL.n_probes, specials=np.array(SMALL_SPECIALS),
        ref_vocab_maps=fh.vocab_maps.numpy(),
        ref_cluster_w_bits=_bits(fh.cluster_linear.weight.detach()),
        ref_sims_bits=np.stack(sims), ref_probes=np.stack(probes),
        ref_tok_greedy=np.array(tok_g),
        ref_tok_tiebreak=np.array(tok_tb), ref_tok_special=np.array(tok_sp),
        ref_tok_dense=dense)


def small_sample(ref_fh, ref_loading, out, draws=20000, temperature=0.8):
    head = make_head(SMALL, seed=11)
    h = make_hidden(2, SMALL.hidden, seed=13)
    fh = _reference_head(ref_fh, ref_loading, head, SMALL.n_probes, None)
    torch.manual_seed(1234)
    counts = np.zeros((2, SMALL.vocab), dtype=np.int64)
    with torch.no_grad():
        for r in range(2):
            x = h[r].view(1, 1, -1)
            for _ in range(draws):
                t = int(fh.get_next_token(x, do_sample=True, temperature=temperature).view(-1)[0])
                counts[r, t] += 1
    np.savez_compressed(os.path.join(out, "small_sample.npz"), hidden_bits=_bits(h),
                        temperature=temperature, draws=draws, counts=counts)


def config_a(ref_fh, ref_loading, out, rows=8):
    shape = LLAMA32_1B
    head = make_head(shape, seed=0)
    h = make_hidden(rows, shape.hidden, seed=1)
    fh = _reference_head(ref_fh, ref_loading, head, shape.n_probes, None)
    sims, probes, toks, tok_g = [], [], [], []
    with torch.no_grad():
        for r in range(rows):
            x = h[r].view(1, 1, -1)
            sims.append(_bits(fh.cluster_linear(x).view(-1)))
            probes.append(np.sort(fh._get_top_clusters(x).view(-1).numpy()))
            tok_g.append(_reference_greedy(fh, x))
            toks.append(int(fh.get_next_token(x, use_identical_tiebreak=True).view(-1)[0]))
    np.savez_compressed(os.path.join(out, "config_a.npz"), hidden_bits=_bits(h),
                        ref_sims_bits=np.stack(sims), ref_probes=np.stack(probes),
                        ref_tok_greedy=np.array(tok_g), ref_tok_tiebreak=np.array(toks))
    with open(os.path.join(out, "config_a.json"), "w") as f:
        json.dump({"shape": shape.__dict__, "head_seed": 0, "hidden_seed": 1, "rows": rows,
                   "checksum": head_checksum(head)}, f, indent=1)


def _top_list(sims_bf16: torch.Tensor, n: int):
    """The n largest bf16 scores of one row (largest first, ties to the smaller
    cluster id) as (uint16 bits, uint16 ids)."""
    v = sims_bf16.float().numpy().astype(np.float64)
    order = np.lexsort((np.arange(v.size), -v))[:n]
    return _bits(sims_bf16[torch.from_numpy(order)]), order.astype(np.uint16)


def batch_reference(ref_fh, ref_loading, out, name, shape, head_seed, hidden_seed, rows=256,
                    extra=64):
    """The reference's stage-1 and greedy outputs on `rows` N(0, 0.25) hidden
    states: probe sets, the top p + extra bf16 scores with their ids (enough
    to judge every cluster within 1e-2 of the p-th score), greedy tokens. The
    hidden states are regenerated from their seed by the tests, so only a
    checksum of them is stored."""
    head = make_head(shape, seed=head_seed)
    h = make_hidden(rows, shape.hidden, seed=hidden_seed)
    fh = _reference_head(ref_fh, ref_loading, head, shape.n_probes, None)
    top_bits, top_ids, probes, toks = [], [], [], []
    t0 = time.time()
    with torch.no_grad():
        for r in range(rows):
            x = h[r].view(1, 1, -1)
            b, i = _top_list(fh.cluster_linear(x).view(-1), shape.n_probes + extra)
            top_bits.append(b)
            top_ids.append(i)
            probes.append(np.sort(fh._get_top_clusters(x).view(-1).numpy()).astype(np.uint16))
            toks.append(_reference_greedy(fh, x))
    print(f"{name}: {rows} reference rows in {time.time() - t0:.0f}s", flush=True)
    np.savez_compressed(os.path.join(out, name + ".npz"), ref_top_bits=np.stack(top_bits),
                        ref_top_ids=np.stack(top_ids), ref_probes=np.stack(probes),
                        ref_tok_greedy=np.array(toks, dtype=np.int64))
    b = h.view(torch.int16).to(torch.int64)  # exact: integer sums of the bf16 bits
    idx = torch.arange(b.numel(), dtype=torch.int64).view_as(b)
    with open(os.path.join(out, name + ".json"), "w") as f:
        json.dump({"shape": shape.__dict__, "head_seed": head_seed, "hidden_seed": hidden_seed,
                   "rows": rows, "checksum": head_checksum(head),
                   "hidden_checksum": [int(b.sum()), int((b * (idx % 65521)).sum())]}, f,
                  indent=1)


def config_b_batch(ref_fh, ref_loading, out):
    """Llama-3.2-1B-shaped head of configs A/B (head seed 0), 256 rows."""
    batch_reference(ref_fh, ref_loading, out, "config_b_batch", LLAMA32_1B, 0, 21)


def config_c_batch(ref_fh, ref_loading, out):
    """Llama-3.1-8B-shaped head of config C (D=4096, head seed 5), 256 rows."""
    batch_reference(ref_fh, ref_loading, out, "config_c_batch", LLAMA31_8B, 5, 22)


def config_d_sample(ref_fh, ref_loading, out, draws_per_row=50000, temperature=0.8):
    """Qwen2.5-1.5B-shaped head, sampling at T=0.8: 2 rows x 50k draws = 1e5."""
    shape = QWEN25_15B
    head = make_head(shape, seed=3)
    h = make_hidden(2, shape.hidden, seed=4)
    fh = _reference_head(ref_fh, ref_loading, head, shape.n_probes, None)
    torch.manual_seed(4321)
    counts = {}
    t0 = time.time()
    with torch.no_grad():
        for r in range(2):
            x = h[r].view(1, 1, -1)
            c = np.zeros(shape.vocab, dtype=np.int64)
            for _ in range(draws_per_row):
                c[int(fh.get_next_token(x, do_sample=True, temperature=temperature).view(-1)[0])] += 1
            counts[r] = c
            print(f"config_d row {r}: {time.time() - t0:.0f}s", flush=True)
    ids = [np.nonzero(counts[r])[0] for r in range(2)]
    np.savez_compressed(os.path.join(out, "config_d_sample.npz"), hidden_bits=_bits(h),
                        temperature=temperature, draws_per_row=draws_per_row,
                        ids0=ids[0], counts0=counts[0][ids[0]],
                        ids1=ids[1], counts1=counts[1][ids[1]])
    with open(os.path.join(out, "config_d_sample.json"), "w") as f:
        json.dump({"shape": shape.__dict__, "head_seed": 3, "hidden_seed": 4,
                   "checksum": head_checksum(head)}, f, indent=1)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default=os.environ.get("FLASHHEAD_REFERENCE_SRC"))
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    if not args.reference_src:
        raise SystemExit("give --reference-src or set FLASHHEAD_REFERENCE_SRC")
    ref_fh, ref_loading = _import_reference(args.reference_src)
    torch.set_num_threads(os.cpu_count())
    jobs = {"small_greedy": small_greedy, "small_sample": small_sample,
            "config_a": config_a, "config_d_sample": config_d_sample,
            "config_b_batch": config_b_batch, "config_c_batch": config_c_batch}
    for name, fn in jobs.items():
        if args.only and name != args.only:
            continue
        t0 = time.time()
        fn(ref_fh, ref_loading, HERE)
        print(f"{name}: {time.time() - t0:.1f}s", flush=True)


if __name__ == "__main__":
    main()
