// The registry of upstream architecture names and the implementations that serve them.
#pragma once
