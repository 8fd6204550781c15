"""PyG-labelled entry points (the reference's GNN_PyG_cuda shims; PyG itself is never imported)."""
