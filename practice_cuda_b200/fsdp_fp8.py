"""FSDP2 all-gather of per-block FP8 weights (the FSDP2 FP8 training config).

A linear weight wrapped in :class:`FP8AllGatherWeight` keeps its
high-precision master values in the FSDP shard, but when FSDP2 unshards it the
shard is first quantized in 128x128 tiles (pcb_quant_per_block) and the
all-gather carries the fp8 bytes plus the fp32 tile scales -- about half the
bytes of a bf16 all-gather.  After the all-gather the unsharded parameter is a
:class:`~practice_cuda_b200.fp8_linear.BlockFP8Weight` that
:class:`~practice_cuda_b200.fp8_linear.FP8BlockLinear` feeds straight into the
FP8 GEMMs.

This is the per-block counterpart of the reference's
``WeightWithDynamicFloat8CastTensor`` FSDP hooks
(``fp8_training/fp8_bench/modules/float8/fsdp_utils.py:271-386``), which
support tensorwise / axiswise scales only (its per-block all-gather is an
``assert False``, ``modules/per_block.py:102-104``).  Per-block scales are local
to a tile, so unlike tensorwise scaling no amax all-reduce is needed; the
only constraint is that every rank's row shard is a whole number of 128-row
tiles (``out_features`` divisible by ``128 * world_size``).
"""

from __future__ import annotations

from typing import Any, Optional

import torch
import torch.nn as nn
from torch.utils._pytree import tree_flatten, tree_map_only

from .fp8_linear import E4M3, BlockFP8Weight, FP8BlockLinear, quantize_weight

# Ops whose tensor outputs stay wrapped (views, copies, new tensors of the
# same role); everything else (optimizer math, reductions) returns plain tensors.
_PRESERVE = {
    torch.ops.aten.empty_like.default,
    torch.ops.aten.new_zeros.default,
    torch.ops.aten.new_empty.default,
    torch.ops.aten.slice.Tensor,
    torch.ops.aten.copy_.default,
    torch.ops.aten.view.default,
    torch.ops.aten.as_strided.default,
    torch.ops.aten._to_copy.default,
    torch.ops.aten._pin_memory.default,
    torch.ops.aten.split.Tensor,
    torch.ops.aten.clone.default,
    torch.ops.aten.detach.default,
    torch.ops.aten.alias.default,
}

# Outputs of these ops alias their input's storage, so the output wrapper
# shares the input's write generation: a write through either invalidates the
# cached quantization of both.
_ALIASING = {
    torch.ops.aten.slice.Tensor,
    torch.ops.aten.view.default,
    torch.ops.aten.as_strided.default,
    torch.ops.aten.split.Tensor,
    torch.ops.aten.detach.default,
    torch.ops.aten.alias.default,
}


class FP8AllGatherWeight(torch.Tensor):
    """High-precision weight whose FSDP2 all-gather is per-block FP8."""

    @staticmethod
    def __new__(cls, tensor: torch.Tensor, pow2: bool = False, gen: Optional[list] = None):
        return torch.Tensor._make_wrapper_subclass(
            cls,
            tensor.size(),
            strides=tensor.stride(),
            storage_offset=tensor.storage_offset(),
            dtype=tensor.dtype,
            layout=tensor.layout,
            device=tensor.device,
            requires_grad=tensor.requires_grad,
        )

    def __init__(self, tensor: torch.Tensor, pow2: bool = False, gen: Optional[list] = None):
        self._tensor = tensor
        self._pow2 = pow2  # power-of-two (E8M0) scales for the block-scaled GEMM
        # Write generation, one cell shared by every wrapper that aliases the
        # same storage (views, .data, .detach()).  The autograd-level version
        # counter does not see writes made through a .data alias (it gets a
        # fresh counter) nor those made below the Python dispatch key, so the
        # cache is keyed on this cell instead.
        self._gen = gen if gen is not None else [0]

    def __repr__(self):
        return f"FP8AllGatherWeight({self._tensor!r})"

    def __tensor_flatten__(self):
        return ["_tensor"], {"pow2": self._pow2}

    @staticmethod
    def __tensor_unflatten__(inner, meta, outer_size, outer_stride):
        return FP8AllGatherWeight(inner["_tensor"], bool(meta and meta.get("pow2")))

    @classmethod
    def __torch_dispatch__(cls, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        wrapped = [t for t in tree_flatten((args, kwargs))[0] if isinstance(t, FP8AllGatherWeight)]
        if func._schema.is_mutable:
            # Any op that may write a weight (optimizer updates, FSDP's
            # copy-in, writes through an alias) invalidates its cached
            # quantization and that of every wrapper aliasing it.
            for t in wrapped:
                t._gen[0] += 1
        pow2 = any(t._pow2 for t in wrapped)
        gen = wrapped[0]._gen if (func in _ALIASING and wrapped) else None
        args, kwargs = tree_map_only(FP8AllGatherWeight, lambda t: t._tensor, (args, kwargs))
        out = func(*args, **kwargs)
        if func not in _PRESERVE:
            return out
        return tree_map_only(torch.Tensor, lambda t: FP8AllGatherWeight(t, pow2, gen), out)

    # ---- FSDP2 all-gather extension -------------------------------------------
    def _quantized_shard(self, world: int):
        """All-gather inputs for the current shard values, cached until the
        shard may have been written, so the backward re-gather and
        :func:`precompute_fp8_block_weights` do not quantize twice.

        The key is the write generation shared by all wrappers of this
        storage (bumped by every mutable op dispatched on any of them,
        including ``w.data.add_`` and ``w.detach().copy_``), the inner
        tensor's own version counter and its storage pointer (FSDP may swap
        the storage)."""
        key = (self._gen[0], self._tensor._version, self._tensor.data_ptr(), world)
        cached = getattr(self, "_fp8_cache", None)
        if cached is not None and cached[0] == key:
            return self._fresh(cached[1], world), cached[2]
        shard = self._tensor.detach()
        data, scale = quantize_weight(shard, pow2=True) if self._pow2 else quantize_weight(shard)
        if world == 1:
            # FSDP2's single-rank path takes exactly one all-gather input, so
            # the scales ride in extra uint8 rows appended to the fp8 rows.
            rows, cols = data.shape
            sbytes = scale.numel() * 4
            extra = (sbytes + cols - 1) // cols
            packed = torch.zeros((rows + extra, cols), dtype=torch.uint8, device=data.device)
            packed[:rows].copy_(data.view(torch.uint8))
            packed[rows:].view(-1)[:sbytes].copy_(scale.reshape(-1).view(torch.uint8))
            inputs, meta = (packed,), {"rows": rows, "scale_shape": tuple(scale.shape)}
        else:
            inputs, meta = (data.view(torch.uint8), scale), None
        self._fp8_cache = (key, inputs, meta)
        return self._fresh(inputs, world), meta

    @staticmethod
    def _fresh(inputs, world):
        # At world size 1 FSDP2 may use the all-gather input itself as the
        # unsharded storage and free it on reshard: hand it a copy.
        return tuple(t.clone() for t in inputs) if world == 1 else inputs

    def fsdp_pre_all_gather(self, mesh, outer_size, outer_stride, module, mp_policy):
        shard = self._tensor
        if shard.shape[0] % 128 != 0:
            raise ValueError(
                f"per-block FP8 all-gather needs whole 128-row tiles per rank; shard has {shard.shape[0]} rows "
                f"(out_features {outer_size[0]} over {mesh.size()} ranks)"
            )
        return self._quantized_shard(mesh.size())

    def fsdp_post_all_gather(
        self,
        all_gather_outputs: tuple[torch.Tensor, ...],
        metadata: Any,
        param_dtype: torch.dtype,
        *,
        out: Optional[torch.Tensor] = None,
    ):
        if metadata is not None:  # single rank: fp8 rows followed by the packed scales
            (packed,) = all_gather_outputs
            rows = metadata["rows"]
            shape = metadata["scale_shape"]
            data_u8 = packed[:rows]
            nbytes = shape[0] * shape[1] * 4
            scale = packed[rows:].reshape(-1)[:nbytes].view(torch.float32).view(shape)
            inner = (packed,)
        else:
            data_u8, scale = all_gather_outputs
            inner = (data_u8, scale)
        data = data_u8.view(E4M3)
        if out is not None:
            # Storage of the inner tensors was re-filled in place by FSDP.
            out._data = data
            out._scale = scale
            return None
        return BlockFP8Weight(data, scale, param_dtype), inner


@torch.no_grad()
def precompute_fp8_block_weights(module: nn.Module) -> int:
    """Quantize every FP8 all-gather weight shard of ``module`` now.

    Call after ``optimizer.step()``: the next FSDP2 unshard (and the backward
    re-gather) then only copies the cached fp8 bytes and scales.  The
    per-block counterpart of the reference's
    ``precompute_bmm_float8_dynamic_scale_for_fsdp``
    (``fp8_training/fp8_bench/modules/bmm_linear.py:676-752``); per-block
    scales are local to a 128x128 tile, so no all-reduce is involved.
    Returns the number of shards quantized.
    """
    count = 0
    for m in module.modules():
        if not isinstance(m, FP8BlockLinear):
            continue
        w = m.weight
        local = getattr(w, "_local_tensor", w)  # DTensor shard under FSDP2
        if isinstance(local, FP8AllGatherWeight):
            mesh = getattr(w, "device_mesh", None)
            local._quantized_shard(mesh.size() if mesh is not None else 1)
            count += 1
    return count


def enable_fp8_all_gather(module: nn.Module) -> nn.Module:
    """Wrap the weight of every :class:`FP8BlockLinear` in ``module`` so that
    FSDP2 all-gathers it as per-block FP8 (call before ``fully_shard``)."""
    for m in module.modules():
        if isinstance(m, FP8BlockLinear) and not isinstance(m.weight, FP8AllGatherWeight):
            m.weight = nn.Parameter(FP8AllGatherWeight(m.weight.data, pow2=m.scaling == "e8m0"),
                                    requires_grad=m.weight.requires_grad)
    return module
