"""B200-native paged KV-cache hot path of mini-infra-qwen3.

Sub-packages mirror the reference's module layout so that code written against
``mini_infra.{core,worker,model,engine}`` ports by changing the package name:

* ``core``   — control plane (requests, scheduler, block tables); pure Python, no torch;
* ``worker`` — ``PagedKVCachePool`` / ``PagedRunner``: the data plane, calling the CUDA library;
* ``model``  — Qwen3 with the paged attention branch routed to the CUDA kernels;
* ``engine`` — ``EngineConfig`` and ``run_scheduler`` for ``paged-kv-cache`` (+ chunked prefill);
* ``ops``    — torch-facing wrappers of the C ABI in ``include/mi_paged.h``.

The CUDA library (``_lib/libmi_paged.so``) is loaded on first use; there is no CPU path.
"""

__version__ = "0.1.0"
