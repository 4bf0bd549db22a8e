from circuit_rag.hierarchy.build import CircuitIndex, build_circuit_index

__all__ = ["CircuitIndex", "build_circuit_index"]
