"""dlvk_b200 subpackage."""
