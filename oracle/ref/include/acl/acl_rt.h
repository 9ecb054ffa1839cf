/* See acl.h: the runtime declarations live there. */
#include "acl/acl.h"
