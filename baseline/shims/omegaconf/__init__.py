"""Minimal OmegaConf stand-in: plain dicts play the role of DictConfig."""

import copy

import yaml

DictConfig = dict
ListConfig = list


class OmegaConf:
    @staticmethod
    def is_config(obj):
        return False

    @staticmethod
    def to_container(cfg, resolve=True):
        return copy.deepcopy(cfg)

    @staticmethod
    def create(obj=None):
        return copy.deepcopy(obj) if obj is not None else {}

    @staticmethod
    def load(path):
        with open(path) as f:
            return yaml.safe_load(f) or {}

    @staticmethod
    def merge(*cfgs):
        out = {}
        for c in cfgs:
            out = _merge(out, c)
        return out


def _merge(a, b):
    out = copy.deepcopy(a)
    for k, v in (b or {}).items():
        out[k] = _merge(out[k], v) if isinstance(v, dict) and isinstance(out.get(k), dict) else copy.deepcopy(v)
    return out
