"""B200-native KG constraint engine: per-decode-step advance and logits masking.

Host API mirrors the reference xgraph package (build_kg_index, KGVersions, Engine,
closed_span); the per-step work runs in hand-written sm_100a CUDA kernels behind a
C ABI (libxgraph_b200.so, declared in include/xgraph_b200.h).
"""

from importlib import import_module

_EXPORTS = {
    "Engine": "engine",
    "EngineUnavailable": "engine",
    "Admission": "engine",
    "closed_span": "engine",
    "Entity": "kg",
    "Relation": "kg",
    "KnowledgeGraph": "kg",
    "KGFormatError": "kg",
    "KGIndex": "index",
    "build_kg_index": "index",
    "build_kg_index_arrays": "index",
    "load_kg_index": "index",
    "save_kg_index": "index",
    "KGVersions": "kgversions",
    "build_kg_versions": "kgversions",
    "ServedTokenizer": "tokenizer",
    "SpanSyntax": "syntax",
    "MatchedExecutor": "programs",
    "MatchedPath": "programs",
}
__all__ = list(_EXPORTS)


def __getattr__(name):
    if name not in _EXPORTS:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    value = getattr(import_module(f".{_EXPORTS[name]}", __name__), name)
    globals()[name] = value
    return value
