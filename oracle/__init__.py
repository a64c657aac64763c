"""ORACLE — test infrastructure, not part of the product.

`oracle` restates go-tensor's reference CPU path so device results can be
checked against it:

* ``cpu_backend.c`` (built to ``_build/liboracle_cpu.so``) restates the pure-Go
  CPU backend, ``internal/cpu/cpu.go`` and ``internal/cpu/linalg.go``;
* ``gotensor_ref.py`` restates the layers above the backend interface
  (``tensor/``, ``nn/``, ``optim/``) over any object with the backend methods.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg import this package.
"""
