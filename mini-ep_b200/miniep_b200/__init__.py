"""miniep_b200: mini-EP's expert-parallel MoE layer as sm_100a CUDA kernels.

Drop-in for the reference's MoE backend (miniep.ep / miniep.modeling):
``Placement``, ``Comm``, ``EPStats``, ``EPMoEBackend``, ``LocalMoEBackend`` and
``plan_balanced`` keep the reference's names, arguments and plan/stats
formats; the layer step runs in libminiep_b200.so (C ABI in
include/miniep_b200.h).
"""
from .ep import (Comm, EPMoEBackend, EPStats, GraphedMoEBlock, LocalMoEBackend,  # noqa: F401
                 Placement, StreamedMoEBlock, router_topk)
from .balancer import layer_imbalance, plan_balanced, plan_lpt, straggler_overhead  # noqa: F401
from ._lib import MEPError  # noqa: F401

__all__ = ["Comm", "EPMoEBackend", "EPStats", "GraphedMoEBlock", "LocalMoEBackend", "Placement",
           "StreamedMoEBlock", "router_topk",
           "plan_balanced", "plan_lpt", "straggler_overhead", "layer_imbalance", "MEPError"]
