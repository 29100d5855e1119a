"""install(): every module of a plastic-infer tree that holds a KV-path name gets ours.

The mechanics are checked on a stand-in package with the reference's module layout
(so the test runs anywhere); when a real plastic-infer source tree is given through
PLASTIC_INFER_SRC, the same check runs on it and its paged runner is driven through
our KV store on CPU bookkeeping.
"""

from __future__ import annotations

import importlib
import os
import sys
import textwrap

import pytest

from plastic_infer_b200 import install as inst
from plastic_infer_b200.exec import attention as our_att
from plastic_infer_b200.exec import runner_paged as our_rp
from plastic_infer_b200.kv import kv_store as our_ks

FAKE_MODULES = {
    "kv/kv_store.py": "class KVConfig: pass\nclass KVPagedStorage: pass\n"
                      "class KVRequestCache: pass\nclass KVStore: pass\n",
    "exec/attention.py": "def gather_paged_kv(): pass\ndef paged_attention_v1(): pass\n"
                         "def host_stream_attention_v1(): pass\n",
    "exec/runner_paged.py": "from .attention import paged_attention_v1\n"
                            "from ..kv.kv_store import KVConfig, KVRequestCache, KVStore\n"
                            "def make_kv_config(): pass\ndef _attn_paged(): pass\n"
                            "def _write_kv_layer(): pass\ndef _allocate_pages_for_tokens(): pass\n",
    "exec/runner_moe_paged.py": "from ..kv.kv_store import KVRequestCache, KVStore\n"
                                "from .runner_paged import (_allocate_pages_for_tokens, _attn_paged,"
                                " _write_kv_layer, make_kv_config)\n",
    "runtime/engine.py": "from ..exec.runner_moe_paged import make_kv_config\n"
                         "from ..kv.kv_store import KVStore\n",
}


@pytest.fixture
def fake_pkg(tmp_path):
    root = tmp_path / "fake_plastic"
    for rel, body in FAKE_MODULES.items():
        p = root / rel
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_text(textwrap.dedent(body))
    for d in ("", "kv", "exec", "runtime"):
        (root / d / "__init__.py").write_text("")
    sys.path.insert(0, str(tmp_path))
    yield "fake_plastic"
    sys.path.remove(str(tmp_path))
    for name in [m for m in sys.modules if m.startswith("fake_plastic")]:
        del sys.modules[name]


def _check(pkg: str, expect_ours: bool) -> None:
    ours = inst._ours()
    for rel, names in inst.TARGETS.items():
        mod = importlib.import_module(f"{pkg}.{rel}")
        for name in names:
            if hasattr(mod, name):
                assert (getattr(mod, name) is ours[name]) == expect_ours, (rel, name)


def test_install_rebinds_every_importer_and_uninstalls(fake_pkg: str) -> None:
    originals = importlib.import_module(f"{fake_pkg}.exec.runner_moe_paged")._attn_paged
    handle = inst.install(fake_pkg)
    _check(fake_pkg, True)
    moe = importlib.import_module(f"{fake_pkg}.exec.runner_moe_paged")
    assert moe._write_kv_layer is our_rp._write_kv_layer
    assert importlib.import_module(f"{fake_pkg}.runtime.engine").KVStore is our_ks.KVStore
    assert importlib.import_module(f"{fake_pkg}.exec.attention").paged_attention_v1 is \
        our_att.paged_attention_v1
    handle.uninstall()
    _check(fake_pkg, False)
    assert moe._attn_paged is originals


@pytest.mark.skipif(not os.environ.get("PLASTIC_INFER_SRC"),
                    reason="set PLASTIC_INFER_SRC to a plastic-infer src/ tree")
def test_install_on_real_reference_tree() -> None:
    sys.path.insert(0, os.environ["PLASTIC_INFER_SRC"])
    sys.dont_write_bytecode = True
    handle = inst.install("plastic_infer")
    try:
        _check("plastic_infer", True)
        import torch

        from plastic_infer.exec.runner_paged import make_kv_config
        from plastic_infer.kv.kv_store import KVStore
        from plastic_infer.exec.runner import ModelConfig

        cfg = ModelConfig(n_layers=2, n_heads=4, n_kv_heads=2, head_dim=8, hidden_dim=32,
                          intermediate_dim=64, vocab_size=50, max_seq_len=64)
        store = KVStore(make_kv_config(cfg, max_pages=32))
        assert isinstance(store, our_ks.KVStore)
        assert store.gpu.k_pages.shape == (32, 2, 8, 16)  # reference logical layout
        cache = store.new_request()
        cache.reserve_tokens(20)
        assert cache.get_block_table_for_layer(0) == [0, 2]
        assert store.gpu.allocator.used_pages == 4
        assert torch.equal(store.gpu.k_phys.permute(0, 1, 3, 2), store.gpu.k_pages)
    finally:
        handle.uninstall()
