/* stub: the reference's oracle does not use half types on the host */
#pragma once
