"""prismyra_b200: the routed-expert MoE layer of Prismyra, rebuilt for B200 (sm_100a).

The compute path is ``libprismyra_moe.so`` (C ABI in ``include/prismyra_moe.h``); this package is its host
side: the ctypes binding (``_lib``), torch-facing calls (``ops``), the adapter registry and drop-in modules
(``kernels``), synthetic inputs (``synth``) and expert parallelism (``ep``).
"""

__version__ = "0.1.0"
