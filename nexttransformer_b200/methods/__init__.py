"""Contributed methods, one package per method, each declared by its ``method.json``.

The packages here are the plugin methods of the reference tree
(``nexttransformer/methods/*``), written against this package's shell: gated attention
(elementwise and headwise), exclusive self attention (XSA), Inkling relative-position logits,
SimpleHC, Full AttnRes with Canon layers, and Multi-Stream Attention Residuals (MSAR).
"""
