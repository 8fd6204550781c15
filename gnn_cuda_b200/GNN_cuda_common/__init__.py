"""Drop-in counterpart of GNN_cuda's ``GNN_cuda_common`` package, backed by libgnnb200.so."""
