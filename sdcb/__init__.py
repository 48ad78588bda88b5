"""Namespace of the B200 GCDRNet backend (``sdcb.gcdrnet_b200``)."""
