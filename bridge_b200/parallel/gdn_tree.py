"""Focused pure-GDN tree executor under head-parallel CP (test-grade).

A residual stack of GDN layers executes one tree: Push stores each layer's
final state graph-free, siblings start from independent anchors of the parent
state, and Pop back-propagates the relayed dState through a recompute.
Parameter versions are checked so an in-place update between Push and Pop is
caught.

Parity: verl/models/mcore/tpr/parallel/gdn_tree.py:13-160.
"""

from __future__ import annotations

import torch
from torch import Tensor, nn

from ..tpr.prefix_state import GDNLayerState, GDNPrefixState
from .gdn_state import forward_gdn_cp_with_state


class GDNCPStack(nn.Module):
    """Residual stack ``x + gdn_i(x)`` of head-parallel GDN layers."""

    def __init__(self, layers: list[nn.Module], cp_group) -> None:
        super().__init__()
        self.layers = nn.ModuleList(layers)
        self.cp_group = cp_group

    def forward(self, x: Tensor, states: dict[int, GDNLayerState] | None, *, capture: bool = True):
        finals = {}
        for i, layer in enumerate(self.layers, start=1):
            y, st = forward_gdn_cp_with_state(layer, x, None if states is None else states.get(i), self.cp_group,
                                              capture_final_state=capture)
            x = x + y
            if st is not None:
                finals[i] = st
        return x, finals


class GDNCPBranchExecutor:
    """Push a parent, run independent children from its anchors, Pop the parent with relayed dState."""

    def __init__(self, stack: GDNCPStack) -> None:
        self.stack = stack
        self.saved: dict[int, GDNPrefixState] = {}
        self._versions: dict[int, tuple[int, ...]] = {}

    def _param_versions(self) -> tuple[int, ...]:
        return tuple(p._version for p in self.stack.parameters())

    def push(self, segment_id: int, x: Tensor, parent: int | None = None) -> None:
        init = None if parent is None else self.saved[parent].layer_states
        with torch.no_grad():
            _, finals = self.stack(x, dict(init) if init else None)
        self.saved[segment_id] = GDNPrefixState.save(segment_id, x.shape[0], finals)
        self._versions[segment_id] = self._param_versions()

    def run_child(self, parent: int, x: Tensor, loss_fn) -> Tensor:
        st = self.saved[parent]
        anchors = st.make_anchors()
        y, _ = self.stack(x, dict(anchors.layer_states), capture=False)
        loss = loss_fn(y)
        loss.backward()
        st.accumulate_anchor_gradients(anchors)
        return loss.detach()

    def pop(self, segment_id: int, x: Tensor, loss_fn, parent: int | None = None) -> Tensor:
        if self._versions.get(segment_id) != self._param_versions():
            raise RuntimeError("parameters changed between Push and Pop")
        st = self.saved.pop(segment_id)
        relayed = st.consume_gradients()
        init = None if parent is None else self.saved[parent].make_anchors()
        y, finals = self.stack(x, None if init is None else dict(init.layer_states))
        roots, grads = [loss_fn(y)], [None]
        for layer, g in relayed.items():
            roots += [finals[layer].conv_state, finals[layer].recurrent_state]
            grads += [g.conv_state, g.recurrent_state]
        torch.autograd.backward(roots, grad_tensors=grads)
        if init is not None:
            self.saved[parent].accumulate_anchor_gradients(init)
        st.release()
        return roots[0].detach()
