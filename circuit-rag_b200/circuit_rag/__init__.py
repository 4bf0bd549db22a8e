"""circuit-b200: exact top-k inner-product search on B200 (sm_100a).

Drop-in for the reference package surface (reference circuit_rag/__init__.py:1-7):
CircuitIndex, build_circuit_index, circuit_search, SearchTrace, CircuitRAG,
SearchResult.  The search path is libcircuit.so (hand-written sm_100a CUDA);
there is no CPU search path.
"""
from circuit_rag.hierarchy.build import CircuitIndex, build_circuit_index
from circuit_rag.search import circuit_search, circuit_search_batch, SearchTrace
from circuit_rag.rag import CircuitRAG, SearchResult

__version__ = "0.1.0"
__all__ = ["CircuitRAG", "SearchResult", "CircuitIndex", "build_circuit_index", "circuit_search", "circuit_search_batch",
           "SearchTrace"]
