"""B200-native tensor-parallel decoder-layer forward for the pythonintern inference engine.

The modules mirror the reference engine's Python API (engine/tensor_parallel/layers.py,
engine/tensor_parallel/comm.py, engine/model/*.py, engine/worker/execution_engine.py);
the compute runs in hand-written sm_100a CUDA kernels reached through the C-ABI
library ``libb2tp.so`` (see ``include/b2tp.h``).  Submodules are imported lazily so
that configuration and workload helpers load without the CUDA library.
"""

__version__ = "0.1.0"
