"""Layer prefetch (reference ``src/prefetch.py``) and the automatic prefetcher.

:class:`PrefetchManager`, :class:`LayerWiseZeroQ` and :func:`create_prefetch_hooks`
keep the reference's API (:23-143, :146-271, :274-307).

:class:`AutoPrefetcher` is what the module wrapper actually uses when
``config.async_gather`` is set (the reference declared the field but never read
it): the first forward pass records the order in which hooked modules run; from
then on, entering module ``i`` starts the asynchronous gathers of modules
``i+1 .. i+prefetch_count`` in forward, and of ``i-1 .. i-prefetch_count`` in
backward.  All ranks see the same module order, so they issue the same
collectives in the same order.
"""

from __future__ import annotations

from collections import deque
from typing import Deque, Dict, List, Optional, Set

import torch

from .coordinator import ZeroQCoordinator, ZeroQParamStatus


def in_backward() -> bool:
    try:
        return torch._C._current_graph_task_id() != -1
    except Exception:  # pragma: no cover
        return False


class PrefetchManager:
    """Layer-indexed asynchronous prefetch of sharded parameters."""

    def __init__(self, coordinator: ZeroQCoordinator, prefetch_count: int = 2):
        self.coordinator = coordinator
        self.prefetch_count = prefetch_count
        self._inflight: Set[int] = set()
        self._prefetch_queue: Deque[int] = deque()
        self._layer_params: Dict[int, List[int]] = {}

    def register_layer(self, layer_idx: int, param_ids: List[int]):
        self._layer_params[layer_idx] = list(param_ids)

    def prefetch_for_layer(self, layer_idx: int):
        if layer_idx not in self._layer_params or layer_idx in self._inflight:
            return
        for pid in self._layer_params[layer_idx]:
            p = self.coordinator._params.get(pid)
            if p is not None and p.status == ZeroQParamStatus.NOT_AVAILABLE:
                self.coordinator.fetch_params([pid], async_op=True)
        self._inflight.add(layer_idx)
        self._prefetch_queue.append(layer_idx)

    def wait_for_layer(self, layer_idx: int):
        if layer_idx not in self._layer_params:
            return
        for pid in self._layer_params[layer_idx]:
            p = self.coordinator._params.get(pid)
            if p is None:
                continue
            if p.status == ZeroQParamStatus.NOT_AVAILABLE:
                self.coordinator.fetch_params([pid], async_op=False)
            p.wait_gather()
        self._inflight.discard(layer_idx)

    def release_layer(self, layer_idx: int):
        if layer_idx in self._layer_params:
            self.coordinator.release_params(self._layer_params[layer_idx])

    def prefetch_ahead(self, current_layer: int):
        for i in range(1, self.prefetch_count + 1):
            self.prefetch_for_layer(current_layer + i)

    def get_stats(self) -> Dict[str, int]:
        return {"inflight_layers": len(self._inflight),
                "registered_layers": len(self._layer_params),
                "prefetch_count": self.prefetch_count}


def _find_layers(model: torch.nn.Module, layer_attr: Optional[str]):
    cands = [layer_attr] if layer_attr else []
    cands += ["layers", "h", "block", "model.layers", "transformer.h", "decoder.layers",
              "encoder.layers"]
    for attr in cands:
        cur = model
        ok = True
        for part in attr.split("."):
            if not hasattr(cur, part):
                ok = False
                break
            cur = getattr(cur, part)
        if ok and isinstance(cur, (torch.nn.ModuleList, list)):
            return attr, cur
    raise ValueError("Could not find layer list. Tried: " + ", ".join(cands) +
                     ". Please specify layer_attr manually.")


class LayerWiseZeroQ:
    """Register each layer's frozen params with a coordinator and prefetch by layer."""

    def __init__(self, model: torch.nn.Module, config=None, layer_attr: str = "layers",
                 prefetch_count: int = 2):
        from ..config import B200_CONFIG

        self.model = model
        self.config = config or B200_CONFIG
        self.coordinator = ZeroQCoordinator(self.config)
        self.prefetch = PrefetchManager(self.coordinator, prefetch_count=prefetch_count)
        self.layer_attr, self._layers = _find_layers(model, layer_attr)
        self._setup_layers()

    def _setup_layers(self):
        seen = set()
        for idx, layer in enumerate(self._layers):
            pids = []
            for mname, mod in layer.named_modules():
                for pname, p in mod.named_parameters(recurse=False):
                    if not p.requires_grad:
                        pids.append(self.coordinator.register_parameter(p, mod, pname).param_id)
                        seen.add(id(p))
            self.prefetch.register_layer(idx, pids)
        embed, output = [], []
        for mname, mod in self.model.named_modules():
            for pname, p in mod.named_parameters(recurse=False):
                if id(p) in seen or p.requires_grad:
                    continue
                seen.add(id(p))
                pid = self.coordinator.register_parameter(p, mod, pname).param_id
                (embed if "embed" in f"{mname}.{pname}".lower() else output).append(pid)
        if embed:
            self.prefetch.register_layer(-1, embed)
        if output:
            self.prefetch.register_layer(len(self._layers), output)

    def partition(self):
        self.coordinator.partition_all()

    def forward_with_prefetch(self, *args, **kwargs):
        self.prefetch.wait_for_layer(-1)
        self.prefetch.prefetch_ahead(0)
        return self.model(*args, **kwargs)

    def get_memory_stats(self):
        return self.coordinator.get_memory_stats()


def create_prefetch_hooks(model: torch.nn.Module, prefetch_manager: PrefetchManager,
                          layer_attr: str = "layers"):
    """Per-layer hooks: wait for the layer, prefetch ahead; release under no_grad."""
    _, layers = _find_layers(model, layer_attr)
    handles = []
    for idx, layer in enumerate(layers):
        def pre(module, inputs, _i=idx):
            prefetch_manager.wait_for_layer(_i)
            prefetch_manager.prefetch_ahead(_i)

        def post(module, inputs, outputs, _i=idx):
            if not torch.is_grad_enabled():
                prefetch_manager.release_layer(_i)

        handles.append(layer.register_forward_pre_hook(pre))
        handles.append(layer.register_forward_hook(post))
    return handles


class AutoPrefetcher:
    """Records hooked-module order on the first forward; prefetches neighbours after."""

    def __init__(self, coordinator: ZeroQCoordinator, module_param_ids: Dict, depth: int):
        self.coordinator = coordinator
        self.module_param_ids = module_param_ids
        self.depth = max(0, int(depth))
        self.order: List[torch.nn.Module] = []
        self._index: Dict[int, int] = {}
        self._recording = True

    def on_forward(self, module):
        if self._recording:
            if id(module) in self._index:
                self._recording = False  # second visit: order complete
            else:
                self._index[id(module)] = len(self.order)
                self.order.append(module)
                return
        if in_backward():
            return  # checkpoint recompute: backward prefetch covers it
        self._prefetch(module, +1)

    def on_backward(self, module):
        self._recording = False
        self._prefetch(module, -1)

    def _prefetch(self, module, step: int):
        i = self._index.get(id(module))
        if i is None:
            return
        for k in range(1, self.depth + 1):
            j = i + step * k
            if 0 <= j < len(self.order):
                pids = self.module_param_ids.get(self.order[j])
                if pids:
                    self.coordinator.fetch_params(pids, async_op=True)
