"""Config-driven cluster launcher (reference ``src/opendipaco/launch/__init__.py``).

``LaunchConfig`` / ``load_config`` describe a run, the ``run_*`` functions stand up
each role from it, and ``opendipaco_b200.launch.cli:main`` is the ``opendipaco``
command (also ``python -m opendipaco_b200.launch``).
"""

from .config import LaunchConfig, backbone_config, diloco_config, dipaco_config, load_config
from .roles import (build_corpus, build_documents, run_coordinator, run_ingest, run_local, run_parameter_server,
                    run_relay, run_scheduler, run_tracker, run_worker_role)

__all__ = ["LaunchConfig", "load_config", "backbone_config", "dipaco_config", "diloco_config", "build_documents",
           "build_corpus", "run_coordinator", "run_scheduler", "run_parameter_server", "run_relay", "run_tracker",
           "run_worker_role", "run_ingest", "run_local"]
