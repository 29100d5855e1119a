"""Drop this package's paged-KV path into an installed plastic-infer.

`install()` rebinds, in every plastic-infer module that holds them, the names of the
KV path to this package's implementations (same signatures):

  plastic_infer.kv.kv_store           KVConfig, KVPagedStorage, KVRequestCache, KVStore
  plastic_infer.exec.attention        gather_paged_kv, paged_attention_v1, host_stream_attention_v1
  plastic_infer.exec.runner_paged     the above it imported, plus make_kv_config, _attn_paged,
                                      _write_kv_layer, _allocate_pages_for_tokens
  plastic_infer.exec.runner_moe_paged KVRequestCache, KVStore and the runner_paged helpers it
                                      imported by name (src/plastic_infer/exec/runner_moe_paged.py:18-28)
  plastic_infer.runtime.engine        KVStore, make_kv_config
                                      (src/plastic_infer/runtime/engine.py:31-36)

Rebinding only the defining modules would not be enough: runner_moe_paged and the
engine imported these names with `from ... import`, so their own module globals are
patched too. The engine, memory planner, streamed weights and MoE expert cache are
untouched. `install()` returns a handle whose `uninstall()` restores the originals.
"""

from __future__ import annotations

import importlib
from dataclasses import dataclass, field


def _ours() -> dict[str, object]:
    from .exec import attention as att
    from .exec import runner_paged as rp
    from .kv import kv_store as ks

    return {
        "KVConfig": ks.KVConfig,
        "KVPagedStorage": ks.KVPagedStorage,
        "KVRequestCache": ks.KVRequestCache,
        "KVStore": ks.KVStore,
        "gather_paged_kv": att.gather_paged_kv,
        "paged_attention_v1": att.paged_attention_v1,
        "host_stream_attention_v1": att.host_stream_attention_v1,
        "make_kv_config": rp.make_kv_config,
        "_attn_paged": rp._attn_paged,
        "_write_kv_layer": rp._write_kv_layer,
        "_allocate_pages_for_tokens": rp._allocate_pages_for_tokens,
    }


# module (relative to the package root) -> names rebound there when present
TARGETS: dict[str, tuple[str, ...]] = {
    "kv.kv_store": ("KVConfig", "KVPagedStorage", "KVRequestCache", "KVStore"),
    "exec.attention": ("gather_paged_kv", "paged_attention_v1", "host_stream_attention_v1"),
    "exec.runner_paged": ("KVConfig", "KVRequestCache", "KVStore", "paged_attention_v1",
                          "make_kv_config", "_attn_paged", "_write_kv_layer",
                          "_allocate_pages_for_tokens"),
    "exec.runner_moe_paged": ("KVRequestCache", "KVStore", "make_kv_config", "_attn_paged",
                              "_write_kv_layer", "_allocate_pages_for_tokens"),
    "runtime.engine": ("KVStore", "make_kv_config"),
}


@dataclass
class Installed:
    saved: list[tuple[object, str, object]] = field(default_factory=list)

    def uninstall(self) -> None:
        for mod, name, old in reversed(self.saved):
            setattr(mod, name, old)
        self.saved.clear()


def install(package: str = "plastic_infer", modules: dict[str, tuple[str, ...]] | None = None
            ) -> Installed:
    """Rebind the KV path of `package` to this implementation; return an undo handle.

    Modules of `package` that fail to import (e.g. the engine without its optional
    dependencies) are skipped; a name is rebound only where the module defines it.
    """
    ours = _ours()
    handle = Installed()
    # Import every target before rebinding anything: a module first imported after
    # its source module was patched would capture our names as its "originals".
    loaded = []
    for rel, names in (modules or TARGETS).items():
        try:
            loaded.append((importlib.import_module(f"{package}.{rel}"), names))
        except ImportError:
            continue
    for mod, names in loaded:
        for name in names:
            if hasattr(mod, name):
                handle.saved.append((mod, name, getattr(mod, name)))
                setattr(mod, name, ours[name])
    return handle
