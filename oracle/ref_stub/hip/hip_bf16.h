/* stub: a 2-byte bf16 holder so the header's declarations compile */
#pragma once
struct __hip_bfloat16 { unsigned short x; };
