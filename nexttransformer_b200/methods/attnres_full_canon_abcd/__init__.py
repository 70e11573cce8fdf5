"""Full AttnRes with Canon layers A-D: the Canon AttnRes trunk with one AttnRes group per layer, so
every sublayer reads each earlier block's output as its own depth source.
Behaviour: ``nexttransformer/methods/attnres_full_canon_abcd/__init__.py:1-16``.
"""
from nexttransformer_b200.methods.attnres_canon_abcd import CanonAttnRes, ffn, frozen, init, mixer  # noqa: F401


class FullCanonAttnRes(CanonAttnRes):
    @staticmethod
    def groups(config):
        return config.n_layer


model = FullCanonAttnRes
