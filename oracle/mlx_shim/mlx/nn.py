"""``mlx.nn`` subset (test infrastructure only): Module, Linear, Embedding,
LayerNorm and silu, eager over the torch-backed ``mlx.core`` shim."""

from __future__ import annotations

import math
from typing import Any

import torch

from . import core as mx


class Module:
    """Parameter container; arrays, modules and lists of them are children."""

    def _children(self):
        for key, value in self.__dict__.items():
            if key.startswith("_"):
                continue
            if isinstance(value, (mx.array, Module)) or (
                isinstance(value, (list, tuple)) and value and all(isinstance(v, (mx.array, Module)) for v in value)
            ):
                yield key, value

    def parameters(self) -> dict[str, Any]:
        out: dict[str, Any] = {}
        for key, value in self._children():
            if isinstance(value, mx.array):
                out[key] = value
            elif isinstance(value, Module):
                out[key] = value.parameters()
            else:
                out[key] = [v.parameters() if isinstance(v, Module) else v for v in value]
        return out

    def trainable_parameters(self) -> dict[str, Any]:
        return self.parameters()

    def update(self, params: dict[str, Any]) -> "Module":
        for key, value in params.items():
            current = getattr(self, key)
            if isinstance(value, dict):
                current.update(value)
            elif isinstance(value, list):
                for index, item in enumerate(value):
                    if isinstance(current[index], Module):
                        current[index].update(item)
                    else:
                        current[index] = item
            else:
                setattr(self, key, value)
        return self

    def eval(self) -> "Module":
        return self

    def __call__(self, *args: Any, **kwargs: Any) -> Any:  # pragma: no cover - abstract
        raise NotImplementedError


class Linear(Module):
    def __init__(self, input_dims: int, output_dims: int, bias: bool = True) -> None:
        scale = math.sqrt(1.0 / input_dims)
        self.weight = mx.random.uniform(-scale, scale, (output_dims, input_dims))
        if bias:
            self.bias = mx.random.uniform(-scale, scale, (output_dims,))

    def __call__(self, x: mx.array) -> mx.array:
        y = x @ self.weight.T
        if "bias" in self.__dict__:
            y = y + self.bias
        return y


class Embedding(Module):
    def __init__(self, num_embeddings: int, dims: int) -> None:
        self.weight = mx.random.normal((num_embeddings, dims), scale=math.sqrt(1.0 / dims))

    def __call__(self, x: mx.array) -> mx.array:
        return mx.array(self.weight._t[x._t.long()])

    def as_linear(self, x: mx.array) -> mx.array:
        return x @ self.weight.T


class LayerNorm(Module):
    def __init__(self, dims: int, eps: float = 1e-5, affine: bool = True, bias: bool = True) -> None:
        self.eps = eps
        if affine:
            self.weight = mx.ones((dims,))
            if bias:
                self.bias = mx.zeros((dims,))

    def __call__(self, x: mx.array) -> mx.array:
        t = x._t
        mean = t.mean(dim=-1, keepdim=True)
        var = ((t - mean) ** 2).mean(dim=-1, keepdim=True)
        y = (t - mean) * torch.rsqrt(var + self.eps)
        if "weight" in self.__dict__:
            y = y * self.weight._t
        if "bias" in self.__dict__:
            y = y + self.bias._t
        return mx.array(y.to(t.dtype))


def silu(x: mx.array) -> mx.array:
    return x * mx.sigmoid(x)
