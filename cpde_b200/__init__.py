"""B200-native cPDE engine: derivative-jet MLP forward/backward, costs, reductions
and RPROP/Adam updates as sm_100a CUDA kernels behind the cPDE wire protocol."""
