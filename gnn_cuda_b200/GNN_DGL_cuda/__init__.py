"""DGL-labelled entry points (the reference's GNN_DGL_cuda shims; DGL itself is never imported)."""
