"""``tutti.storage.tutti_nvme.preset_derive``: drive facts from daemon configs (tutti_b200's ``storage.preset``)."""
from tutti_b200.storage.preset import daemon_config_paths, load_daemon_devices, prepare_preset  # noqa: F401
