"""Asynchronous / distributed DiLoCo control plane (reference ``src/opendipaco/schedule/__init__.py``).

* ``AsyncScheduler`` -- in-process fault-tolerant generations over a thread pool.
* ``CoordinatorServer`` / ``run_worker`` -- one coordinator owns weights, TCP workers.
* ``Scheduler`` / ``ParameterServer`` / ``run_sharded_worker`` -- a weight-less
  scheduler, module keys sharded over owners, signed single-use grants.
* ``run_decentralized_worker`` + ``Tracker`` + epochs -- scheduler-less operation.

The tensor work of this package (quantised codecs, robust aggregation, routing)
runs in the sm_100a kernels of ``opendipaco_b200._C`` when tensors are on a GPU.
"""

from .aggregate import AGGREGATES, robust_delta
from .assignment import (assignee, coordinator_key, is_assignee, path_primary, rank_workers, responsible_rank,
                         version_lag)
from .distributed import CoordinatorServer, run_worker
from .identity import PeerIdentity, peer_id_of, sign_record, verify_record
from .observability import MetricsExporter, MetricsLogger
from .ownership import (EpochManager, derive_epoch, make_epoch_record, owner_addr, owner_addrs, owner_eligible,
                        owners_for, rank_owners, verify_epoch_record)
from .quorum import confirm_version, divergent_peers, read_quorum_versions
from .ratelimit import RateLimiter
from .reactor import TransportMetrics
from .reputation import Reputation
from .scheduler import AsyncScheduler, Contribution, Preempt, TransientFault
from .sharded import (ParameterServer, Scheduler, assign_shards, grant_signed_by, make_grant,
                      run_decentralized_worker, run_sharded_worker, verify_grant)
from .tls import client_context, generate_selfsigned_cert, server_context
from .tracker import (Tracker, deregister_peer, fetch_directory, fetch_directory_multi, get_epoch, import_records,
                      make_peer_record, put_epoch, register_peer)

__all__ = [
    "AsyncScheduler", "Contribution", "Preempt", "TransientFault", "CoordinatorServer", "TransportMetrics",
    "run_worker", "Scheduler", "ParameterServer", "run_sharded_worker", "run_decentralized_worker",
    "assign_shards", "make_grant", "verify_grant", "grant_signed_by", "server_context", "client_context",
    "generate_selfsigned_cert", "MetricsExporter", "MetricsLogger", "robust_delta", "AGGREGATES", "Reputation",
    "RateLimiter", "PeerIdentity", "peer_id_of", "sign_record", "verify_record", "Tracker", "make_peer_record",
    "register_peer", "deregister_peer", "fetch_directory", "fetch_directory_multi", "import_records", "put_epoch",
    "get_epoch", "owner_eligible", "owner_addr", "owner_addrs", "EpochManager", "rank_owners", "owners_for",
    "make_epoch_record", "verify_epoch_record", "derive_epoch", "rank_workers", "responsible_rank", "assignee",
    "is_assignee", "version_lag", "coordinator_key", "path_primary", "confirm_version", "divergent_peers",
    "read_quorum_versions",
]
