"""B200-native (sm_100a) paged/packed attention hot path for the llm-engineering engine.

The reference engine keeps its block pool, scheduler, ``ModelRunner`` protocol and
Hugging Face hooks; this package supplies the path underneath them:

* ``ops``      — torch-facing wrappers of the C-ABI kernels (K1 KV write, K2 decode,
                 K3 prefill, K4 metadata) in ``libb200paged.so``.
* ``storage``  — ``PagedKVStorage`` with the reference's layout and errors, writing
                 through K1.
* ``engine``   — the host-side engine bookkeeping (requests, sequences, block pool,
                 scheduler, sampler, engine loop) with the reference's interfaces.
* ``runner``   — ``B200PagedModelRunner`` (the ``ModelRunner`` drop-in), its HF cache
                 and registered attention function.
* ``replicas`` — data-parallel engine replicas, one process per GPU.

The directory name contains a hyphen, so it is imported under the module name
``llm_engineering_b200`` (``__graft_entry__.load_package()`` registers it).
"""

__version__ = "0.1.0"
