"""B200-native (sm_100a) forward pass of the pre-norm Transformer layer stack
of torch_transformer_benchmark.py, behind the reference's drop-in surface."""
__version__ = "0.1.0"
