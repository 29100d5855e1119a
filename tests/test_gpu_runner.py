"""End-to-end C1 parity: the tiny Qwen3-architecture decoder.

The reference ran prefill_forward_paged + 32 greedy decode_step_paged steps for 4
ragged prompts (fp32, CPU) and stored tokens and logits (golden c1_tiny.npz). Here
the same weights run on the GPU through this package's runner, whose KV writes and
decode attention are the sm_100a kernels. Decoding is teacher-forced with the
reference tokens, so every step's logits are comparable even where the reference's
top-2 logits nearly tie; the greedy token must agree wherever the reference margin
is clear.
"""

from __future__ import annotations

import pathlib

import numpy as np
import pytest
import torch

from plastic_infer_b200.decode import BatchTables, decode_step_paged_batched
from plastic_infer_b200.exec.runner import DenseWeights, ModelConfig
from plastic_infer_b200.exec.runner_paged import (decode_step_paged, make_kv_config,
                                                  prefill_forward_paged)
from plastic_infer_b200.kv import KVStore
from tests.golden.inputs import C1_MODEL, c1_weights

pytestmark = pytest.mark.gpu
GOLD = pathlib.Path(__file__).resolve().parent / "golden"
DEV = torch.device("cuda", 0)
LOGIT_ATOL = 2e-3
MARGIN = 1e-2


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLD / "c1_tiny.npz")


@pytest.fixture(scope="module")
def model():
    cfg = ModelConfig(**C1_MODEL, dtype=torch.float32)
    w = DenseWeights({k: torch.from_numpy(v).to(DEV) for k, v in c1_weights().items()})
    return cfg, w


def _prompts(g) -> list[list[int]]:
    out, cur = [], 0
    for n in g["prompt_lens"]:
        out.append([int(t) for t in g["prompts"][cur:cur + n]])
        cur += n
    return out


def _check_step(g, r: int, step: int, logits: torch.Tensor) -> None:
    lg = logits.float().cpu().numpy()
    ref_tok = int(g["tokens"][r, step])
    if g["margins"][r, step] > MARGIN:
        assert int(lg.argmax()) == ref_tok, (r, step)
    steps = list(g["logit_steps"])
    if step in steps:
        ref = g["logits"][r, steps.index(step)]
        err = np.abs(lg - ref).max()
        assert err < LOGIT_ATOL, f"request {r} step {step}: max |dlogit| {err:.2e}"


def test_c1_sequential_api_matches_reference(golden, model) -> None:
    cfg, w = model
    store = KVStore(make_kv_config(cfg, max_pages=256, max_host_chunks=8, device=DEV))
    for r, prompt in enumerate(_prompts(golden)):
        cache = store.new_request()
        logits = prefill_forward_paged(w, cfg, store, cache, torch.tensor(prompt, device=DEV))
        _check_step(golden, r, 0, logits)
        for step in range(1, golden["tokens"].shape[1]):
            logits = decode_step_paged(w, cfg, store, cache, int(golden["tokens"][r, step - 1]))
            _check_step(golden, r, step, logits)


def test_c1_batched_decode_matches_reference(golden, model) -> None:
    cfg, w = model
    store = KVStore(make_kv_config(cfg, max_pages=256, max_host_chunks=8, device=DEV))
    prompts = _prompts(golden)
    caches = []
    for r, prompt in enumerate(prompts):
        cache = store.new_request()
        logits = prefill_forward_paged(w, cfg, store, cache, torch.tensor(prompt, device=DEV))
        _check_step(golden, r, 0, logits)
        caches.append(cache)
    tables = BatchTables(store, caches)
    for step in range(1, golden["tokens"].shape[1]):
        ids = [int(golden["tokens"][r, step - 1]) for r in range(len(caches))]
        logits = decode_step_paged_batched(w, cfg, store, caches, ids, tables)
        for r in range(len(caches)):
            _check_step(golden, r, step, logits[r])
