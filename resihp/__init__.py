"""resihp: a resilient hybrid-parallel (TP x PP x DP) training runtime for B200.

Pure planning (``config``, ``memory``, ``planner``, ``plan``) is torch-free; the
runtime (``parallel``, ``recovery``, ``control``, ``membership``, ``launch``,
``train``) drives a Llama-style or GPT-2-style decoder through hand-written sm_100a
kernels (``ops``) on CUDA and plain torch on CPU.
"""

__version__ = "0.1.0"
