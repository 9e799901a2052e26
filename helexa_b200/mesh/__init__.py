"""Peripheral services of the mesh: the federation router in front of several
operators' gateways, the SSRF-guarded tool fetcher, the account ledger service and the
continuous benchmark daemon."""
