"""The ``tutti`` import path of tutti_b200, so deployments configured for Tutti keep their paths.

vLLM configs name the connector by module path
(``"kv_connector_module_path": "tutti.integration.vllm.connector"``); that module and
the engine/store/index classes a Tutti user imports resolve to tutti_b200's
implementations here. Constructor options follow tutti_b200 (see each class).
"""
