"""Drop-in counterparts of HELM's helm.runtime KV-cache modules."""
